// Opt-in per-row scale search for the fixed-step E8 quantizer (no
// counterpart in the reference: qlab.py:159-183 uses one global step).
//
// For every row of the rotated matrix and each of 16 candidate steps
// step_c = step * 2^((c - 8) / 8), the row is decoded exactly as q_e8_fast
// decodes it (per-256 group RMS in numpy's pairwise order, gn = g / rms,
// p = e8_decode(gn / step_c), rec = (p * step_c) * rms) and two numbers are
// kept:
//   D[r][c]  sum of (A - rec)^2 over the row: each group's 256 squares in
//            numpy's pairwise order, then the row's groups in numpy order;
//   H[r][c]  N log2 N - sum_v cnt_v log2 cnt_v, the bits of the row's N
//            lattice coordinates z = 2p under their own histogram, summed
//            over z = -255 .. 255 in order with log2 from a host table.
// The host then picks, per row, the first argmin over c of D + lam * H at
// the smallest lam (bisection in exact midpoints) whose total rate
// sum_r H[r][c_r] is at most the global step's (c = 8), and a second kernel
// decodes every row at its chosen step.  Every operation is one IEEE fp64
// operation in a fixed order, so the result equals the oracle's restatement
// (oracle/uq_oracle.py e8_scale_search) bit for bit.
#include <cuda_runtime.h>

#include <cmath>
#include <vector>

#include "uq_common.cuh"
#include "uq_e8core.cuh"
#include "uq_groupsum.cuh"

namespace {

constexpr int kCand = 16;
constexpr int kBase = 8;           // the candidate equal to the given step
constexpr int kZMax = 255;         // |2p| bound of the rate histogram
constexpr int kBins = 2 * kZMax + 1;
constexpr int kGroup = 256;
constexpr int kWarps = 8;

// 2^((c - 8) / 8), c = 0 .. 15 (the oracle's E8_SEARCH_FACTORS)
const double kFactor[kCand] = {
    0x1.0000000000000p-1, 0x1.172b83c7d517bp-1, 0x1.306fe0a31b715p-1, 0x1.4bfdad5362a27p-1,
    0x1.6a09e667f3bcdp-1, 0x1.8ace5422aa0dbp-1, 0x1.ae89f995ad3adp-1, 0x1.d5818dcfba487p-1,
    0x1.0000000000000p+0, 0x1.172b83c7d517bp+0, 0x1.306fe0a31b715p+0, 0x1.4bfdad5362a27p+0,
    0x1.6a09e667f3bcdp+0, 0x1.8ace5422aa0dbp+0, 0x1.ae89f995ad3adp+0, 0x1.d5818dcfba487p+0};
__constant__ double c_factor[kCand];

// Lattice point of the 8-vector a of a group with RMS r at step s: the
// fp32 screen of the fixed-step kernels when every decision clears its
// margin, else the exact fp64 decode of (a / r) / s.  All-zero vectors keep
// their signed zeros.
__device__ __forceinline__ void decode_at(const double (&a)[8], double r, double s, double (&p)[8]) {
    const double rs = d_mul(r, s);
    const float inv = rs >= 0x1p-100 ? float(1.0 / rs) : __int_as_float(0x7fc00000);
    float y32[8];
    float ymax = 0.f;
    bool fin = true, zero = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        y32[i] = __fmul_rn(float(a[i]), inv);
        ymax = fmaxf(ymax, fabsf(y32[i]));
        fin &= isfinite(y32[i]);
        zero &= a[i] == 0.0;
    }
    const float M = __fadd_rn(__fmul_rn(ymax, 0x1p-21f), 0x1p-40f);
    if (zero) {
#pragma unroll
        for (int i = 0; i < 8; ++i) p[i] = a[i];
    } else if (!(fin && ymax < 0x1p20f && e8_screen(y32, M, p))) {
        double y[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = (a[i] / r) / s;
        e8_point(y, p);
    }
}

// Loads the lane's 8-vector at e0 (zeros past the row).  NC: through the
// read-only path (only where the kernel writes no output over the input).
template <bool NC>
__device__ __forceinline__ void load8(const double *row, int64_t e0, int n, double (&a)[8]) {
    if (e0 + 8 <= n) {
        const double2 *q = reinterpret_cast<const double2 *>(row + e0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const double2 t = NC ? __ldg(q + i) : q[i];
            a[2 * i] = t.x;
            a[2 * i + 1] = t.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) a[i] = 0.0;
    }
}

// Position of element e of a unit in the warp's slab: e ^ ((e >> 4) & 15).
// The squared errors are written with lane v at e = 8 v + i (i fixed per
// store) and read by warp_group_sumsq with four runs of 8 consecutive
// elements 128 apart; with this swizzle both touch each of the 16 bank pairs
// exactly twice (two wavefronts per 8-byte warp access, the minimum), where
// the plain layout took 16 and 4.
__device__ __forceinline__ int slab_pos(int e) { return e ^ ((e >> 4) & 15); }

// One CTA per (row, candidate): D and H of that pair.  CTA b takes row
// b / 16 and candidate b % 16, so a row's 16 CTAs run together and read it
// from L2 once it is there.  Warps walk units of two groups (the warp layout
// of WarpGroup<256>); the squared errors of a unit go through a warp slab in
// shared memory so that their sums take numpy's order.
__global__ void __launch_bounds__(kWarps * 32) e8_search_kernel(const double *A, int n, double step,
                                                                  const double *LG, double *D, double *H,
                                                                  int *bad) {
    using W = WarpGroup<kGroup>;
    __shared__ __align__(16) double slab[kWarps][2 * kGroup];
    __shared__ double dg[4096 / kGroup * 32];      // per-group sums (n <= 2^17)
    __shared__ int hist[kBins];
    const int row = int(blockIdx.x / kCand), c = int(blockIdx.x % kCand);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const double s = d_mul(step, c_factor[c]);
    const double *rowA = A + int64_t(row) * n;
    const int G = n / kGroup, units = (G + 1) / 2;
    for (int i = threadIdx.x; i < kBins; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int u = warp; u < units; u += kWarps) {
        const int64_t e_base = int64_t(u) * 2 * kGroup;
        const double ss = warp_group_sumsq<kGroup, double>(
            [&](int i) -> double { return e_base + i < n ? __ldg(rowA + e_base + i) : 0.0; });
        const double rms = d_add(sqrt(ss / double(kGroup)), 1e-12);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int vv = lane + 32 * h;                 // vector of the unit
            const double r = __shfl_sync(0xffffffffu, rms, h * W::LPG);
            const int64_t e0 = e_base + 8 * vv;
            double a[8], p[8];
            load8<true>(rowA, e0, n, a);
            decode_at(a, r, s, p);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                slab[warp][slab_pos(8 * vv + i)] = d_sub(a[i], d_mul(d_mul(p[i], s), r));
                if (e0 < n) {
                    const int z = int((long long)d_mul(p[i], 2.0));
                    if (z < -kZMax || z > kZMax) atomicExch(bad, 1);
                    else atomicAdd(&hist[z + kZMax], 1);
                }
            }
        }
        __syncwarp();
        const double dsum = warp_group_sumsq<kGroup, double>([&](int i) -> double { return slab[warp][slab_pos(i)]; });
        if (lane == 0) dg[2 * u] = dsum;
        if (lane == W::LPG && 2 * u + 1 < G) dg[2 * u + 1] = dsum;
        __syncwarp();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        D[int64_t(row) * kCand + c] = pairwise_sum<double>([&](int64_t i) { return dg[i]; }, G);
        double acc = 0.0;
        for (int v = 0; v < kBins; ++v) {
            const int k = hist[v];
            acc = d_add(acc, d_mul(double(k), __ldg(LG + k)));
        }
        H[int64_t(row) * kCand + c] = d_sub(d_mul(double(n), __ldg(LG + n)), acc);
    }
}

// Decodes every row at its chosen step: rec = (p * s_r) * rms, idx = 2p.
// rec may be A itself: a lane writes only its own vector, after every lane
// of the warp has read the unit (plain loads, no read-only path).
__global__ void __launch_bounds__(kWarps * 32) e8_rowstep_kernel(const double *A, int n, double step,
                                                                   const int *choice, double *rec, int16_t *idx) {
    using W = WarpGroup<kGroup>;
    const int row = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const double s = d_mul(step, c_factor[choice[row]]);
    const double *rowA = A + int64_t(row) * n;
    const int G = n / kGroup, units = (G + 1) / 2;
    for (int u = warp; u < units; u += kWarps) {
        const int64_t e_base = int64_t(u) * 2 * kGroup;
        const double ss = warp_group_sumsq<kGroup, double>(
            [&](int i) -> double { return e_base + i < n ? rowA[e_base + i] : 0.0; });
        const double rms = d_add(sqrt(ss / double(kGroup)), 1e-12);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int vv = lane + 32 * h;
            const double r = __shfl_sync(0xffffffffu, rms, h * W::LPG);
            const int64_t e0 = e_base + 8 * vv;
            if (e0 >= n) continue;
            double a[8], p[8];
            load8<false>(rowA, e0, n, a);
            decode_at(a, r, s, p);
            const int64_t o = int64_t(row) * n + e0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (rec) rec[o + i] = d_mul(d_mul(p[i], s), r);
                if (idx) idx[o + i] = (int16_t)(long long)d_mul(p[i], 2.0);
            }
        }
    }
}

struct SearchWs {
    double *D, *H, *LG;
    int *choice, *bad;
    size_t bytes;
};

SearchWs carve_search(void *base, int64_t rows, int64_t n) {
    uq::Carver c(base, ~size_t(0));
    SearchWs w{};
    w.D = c.take<double>(size_t(rows) * kCand);
    w.H = c.take<double>(size_t(rows) * kCand);
    w.LG = c.take<double>(size_t(n) + 1);
    w.choice = c.take<int>(size_t(rows));
    w.bad = c.take<int>(1);
    w.bytes = c.off;
    return w;
}

}  // namespace

namespace uq {

size_t e8_search_ws_bytes(int64_t rows, int64_t n) { return carve_search(nullptr, rows, n).bytes; }

// The search on the rotated matrix A (rows, n) fp64; see the file comment.
// Synchronises the stream (the choice of lam is made on the host).
int e8_scale_search(const double *A, int64_t rows, int64_t n, double step, double *rec, int16_t *idx,
                    int32_t *choice_out, double *lam_host, void *ws, size_t ws_bytes, cudaStream_t st) {
    NvtxRange _r("e8_scale_search");
    if (rows == 0) {
        if (lam_host) *lam_host = 0.0;
        return UQ_OK;
    }
    if (rows > ((int64_t(1) << 31) - 1) / kCand)
        return fail(UQ_ERR_UNSUPPORTED, "e8 scale search: %lld rows exceed the grid of 16 CTAs per row", (long long)rows);
    const SearchWs w = carve_search(ws, rows, n);
    if (ws_bytes < w.bytes) return fail(UQ_ERR_WORKSPACE, "e8 scale search: workspace %zu < %zu", ws_bytes, w.bytes);
    // the candidate table lives in each device's constant memory
    if (cudaMemcpyToSymbolAsync(c_factor, kFactor, sizeof(kFactor), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return check_cuda("e8 scale search: candidate table");
    // log2 of the integers 0 .. n from the C library (log2(0) stands for 0)
    std::vector<double> lg(size_t(n) + 1, 0.0);
    for (int64_t i = 1; i <= n; ++i) lg[size_t(i)] = std::log2(double(i));
    if (cudaMemcpyAsync(w.LG, lg.data(), lg.size() * sizeof(double), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemsetAsync(w.bad, 0, sizeof(int), st) != cudaSuccess)
        return check_cuda("e8 scale search: tables");
    {
        ProfScope _p("e8_search", st);
        e8_search_kernel<<<unsigned(rows * kCand), kWarps * 32, 0, st>>>(A, int(n), step, w.LG, w.D, w.H, w.bad);
    }
    int rc = check_cuda("e8_search_kernel launch");
    if (rc) return rc;
    std::vector<double> D(size_t(rows) * kCand), H(size_t(rows) * kCand);
    int bad = 0;
    if (cudaMemcpyAsync(D.data(), w.D, D.size() * sizeof(double), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaMemcpyAsync(H.data(), w.H, H.size() * sizeof(double), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaMemcpyAsync(&bad, w.bad, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return check_cuda("e8 scale search: read tables");
    if (bad) return fail(UQ_ERR_UNSUPPORTED, "e8 scale search: a lattice coordinate 2p lies beyond +-%d", kZMax);
    // per-row choice at lam: first argmin of D + lam * H (one multiply, one add)
    std::vector<int> pick(static_cast<size_t>(rows));
    auto choose = [&](double lam) {
        double total = 0.0;
        for (int64_t r = 0; r < rows; ++r) {
            const double *d = &D[size_t(r) * kCand], *h = &H[size_t(r) * kCand];
            int best = 0;
            double bj = d[0] + lam * h[0];
            for (int c = 1; c < kCand; ++c) {
                const double j = d[c] + lam * h[c];
                if (j < bj) { bj = j; best = c; }
            }
            pick[size_t(r)] = best;
            total += h[best];
        }
        return total;
    };
    double r0 = 0.0;
    for (int64_t r = 0; r < rows; ++r) r0 += H[size_t(r) * kCand + kBase];
    double lam = 0.0;
    if (choose(0.0) > r0) {
        double hi = 1.0;
        for (int i = 0; i < 400 && choose(hi) > r0; ++i) hi *= 2.0;
        double lo = 0.0;
        for (int i = 0; i < 64; ++i) {
            const double mid = (lo + hi) * 0.5;
            if (choose(mid) <= r0) hi = mid;
            else lo = mid;
        }
        lam = hi;
        choose(lam);
    }
    if (lam_host) *lam_host = lam;
    int *dchoice = choice_out ? reinterpret_cast<int *>(choice_out) : w.choice;
    if (cudaMemcpyAsync(dchoice, pick.data(), pick.size() * sizeof(int), cudaMemcpyHostToDevice, st) != cudaSuccess)
        return check_cuda("e8 scale search: choice");
    if (rec || idx) {
        ProfScope _p("e8_rowstep", st);
        e8_rowstep_kernel<<<unsigned(rows), kWarps * 32, 0, st>>>(A, int(n), step, dchoice, rec, idx);
    }
    rc = check_cuda("e8_rowstep_kernel launch");
    if (rc) return rc;
    // the host vector `pick` must outlive the copy
    if (cudaStreamSynchronize(st) != cudaSuccess) return check_cuda("e8 scale search: sync");
    return UQ_OK;
}

}  // namespace uq

extern "C" {

size_t uq_e8_scale_search_workspace_bytes(int64_t rows, int64_t n) {
    if (rows < 0 || n < kGroup) return 0;
    return uq::e8_search_ws_bytes(rows, n);
}

int uq_e8_scale_search(const double *A, int64_t rows, int64_t n, double step, double *rec, int16_t *idx,
                       int32_t *choice, double *lam_host, void *workspace, size_t workspace_bytes, void *stream) {
    if (rows < 0 || n < kGroup || n % kGroup || n > (int64_t(1) << 17) || rows > (int64_t(1) << 31) - 1)
        return uq::fail(UQ_ERR_INVALID,
                        "uq_e8_scale_search: need rows >= 0 and n a multiple of 256 in [256, 2^17] (n=%lld)",
                        (long long)n);
    if (!(step > 0.0) || !std::isfinite(step)) return uq::fail(UQ_ERR_INVALID, "uq_e8_scale_search: step must be > 0");
    if (rows == 0) {
        if (lam_host) *lam_host = 0.0;
        return UQ_OK;
    }
    if (!A || !workspace) return uq::fail(UQ_ERR_INVALID, "uq_e8_scale_search: null pointer");
    if ((reinterpret_cast<uintptr_t>(A) & 15) != 0)
        return uq::fail(UQ_ERR_INVALID, "uq_e8_scale_search: A must be 16-byte aligned");
    return uq::e8_scale_search(A, rows, n, step, rec, idx, choice, lam_host, workspace, workspace_bytes,
                               UQ_STREAM(stream));
}

}  // extern "C"
