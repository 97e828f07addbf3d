// Finite-codebook E8 quantizer (qlab.py:185-198, the labs' q_e8) for sm_100a.
//
// Reference: the flattened A (fp64, zero-padded to whole groups of `group`),
// s = sqrt(mean(g^2)) + 1e-12 per group, gn = g / s as 8-vectors, the nearest
// codeword of cb (scipy cKDTree, exact Euclidean nearest neighbour) and
// out = cb[nearest] * s.  cb (e8_codebook, qlab.py:111-124) is the K points of
// smallest norm of a grid of D8 u (D8 + 1/2) -- coordinates in [-3, 3], resp.
// [-2.5, 3.5] -- each divided by one scale c; the host builds it (its order
// among equal norms is numpy's argsort's) and passes c and the boundary norm.
//
// Three passes over the vectors:
//  1. classify, one thread per vector: gn in fp64, then the E8 point p nearest
//     to gn * c from the fp32 screen (every decision of the closed-form decode
//     clears a proven margin, so p is the unique nearest lattice point).  When
//     p lies in the grid with a norm below the boundary norm it is a codeword,
//     hence the nearest one: out = RN(p / c) * s, the reference's arithmetic.
//     Other vectors are appended to list 1.
//  2. search, list 1: fp32 distances to all K codewords (staged through shared
//     memory, two vectors per thread), keeping the smallest two.  When they
//     differ by more than twice the fp32 error bound (below), the smallest is
//     the exact nearest codeword; the rest go to list 2.
//  3. exact, list 2 (one CTA per vector): fp64 distances sum_i (gn_i - cb_i)^2
//     in coordinate order to all K codewords; the smallest, lowest index on
//     equal distances.  Only here can the choice differ from cKDTree's, whose
//     order of summation and tie rule are its own (an exact fp64 tie, or two
//     distances within fp64 rounding of each other).
//
// fp32 error bound of pass 2: with u = 2^-24, g = RN32(gn), c = RN32(cb),
// e = RN(g - c) is within 2u(1+u)(|gn_i| + |cb_i|) of gn_i - cb_i, and the
// sum of squares (one product, three FMAs per lane pair, one final add) adds
// at most 5u relative, so |d32 - D| <= 18u (|gn|^2 + |cb|^2) (1 + O(u)); two
// codewords are told apart when their d32 differ by more than
// 36u (|gn|^2 + max|cb|^2) < 2^-18 (|gn|^2 + max|cb|^2), the margin used.
#include <cuda_runtime.h>

#include <algorithm>
#include <stdint.h>

#include "uq_common.cuh"
#include "uq_e8core.cuh"

namespace uq {
int e8_quant(const void *A, int a_dtype, int64_t size, int64_t group, double step, double *rec,
             int16_t *idx, double *rms_out, cudaStream_t st);
}

namespace {

typedef unsigned long long u64;

__device__ __forceinline__ u64 pk2(float lo, float hi) {
    u64 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void up2(u64 v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ u64 sub2(u64 a, u64 b) {
    u64 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ u64 mul2(u64 a, u64 b) {
    u64 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c) {
    u64 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ void lds2x64(unsigned addr, u64 &a, u64 &b) {
    asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr));
}

struct QE8Args {
    const void *A;
    int64_t size;          // valid elements
    int64_t group;
    int64_t nvec;          // padded size / 8
    const double *rms;     // per group
    const double *cb;      // K x 8
    const float *cb32;     // K x 8
    int64_t K;
    double scale;          // c: codeword = lattice point / c
    double norm_cut;       // every grid point of lattice norm below this is a codeword (0: none known)
    double *out;           // size
    unsigned *list1, *list2;
    unsigned *cnt;         // [0] list 1 length, [1] list 2 length, [2] non-finite seen, [3] max |cb32|^2 bits
};

// gn of vector v in fp64 (qlab.py:193-194) and each element's group scale.
template <typename TIn>
__device__ __forceinline__ bool load_gn(const QE8Args &a, int64_t v, double gn[8], double s[8]) {
    const TIn *A = static_cast<const TIn *>(a.A);
    bool fin = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t e = 8 * v + i;
        const double x = e < a.size ? double(__ldg(A + e)) : 0.0;
        s[i] = __ldg(a.rms + e / a.group);
        gn[i] = x / s[i];
        fin &= isfinite(gn[i]);
    }
    return fin;
}

// out = cb_value * s for the valid elements of vector v
__device__ __forceinline__ void store_rec(const QE8Args &a, int64_t v, const double c[8], const double s[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t e = 8 * v + i;
        if (e < a.size) a.out[e] = d_mul(c[i], s[i]);
    }
}

// Appends v to a list; one atomic per warp.
__device__ __forceinline__ void append(unsigned *list, unsigned *count, bool want, unsigned v) {
    const unsigned m = __ballot_sync(0xffffffffu, want);
    if (!m) return;
    const int lane = threadIdx.x & 31, leader = __ffs(m) - 1;
    unsigned base = 0;
    if (lane == leader) base = atomicAdd(count, unsigned(__popc(m)));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (want) list[base + __popc(m & ((1u << lane) - 1u))] = v;
}

__global__ void cb_norm_kernel(const float *cb32, int64_t K, unsigned *cnt) {
    float mx = 0.f;
    for (int64_t j = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; j < K; j += int64_t(gridDim.x) * blockDim.x) {
        float n2 = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float c = __ldg(cb32 + 8 * j + i);
            n2 = fmaf(c, c, n2);
        }
        mx = fmaxf(mx, n2);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    // non-negative floats order as their bit patterns
    if ((threadIdx.x & 31) == 0) atomicMax(cnt + 3, __float_as_uint(mx));
}

// Pass 1.  The whole loop body runs for every lane (list appends are warp-wide).
template <typename TIn>
__global__ void __launch_bounds__(256) qe8_classify_kernel(QE8Args a) {
    const float c32 = float(a.scale);
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    const int64_t v_end = (a.nvec + 31) / 32 * 32;
    for (int64_t v = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; v < v_end; v += stride) {
        const bool live = v < a.nvec;
        bool pending = false;
        if (live) {
            double gn[8], s[8];
            const bool fin = load_gn<TIn>(a, v, gn, s);
            if (!fin) {
                atomicExch(a.cnt + 2, 1u);
            } else {
                bool done = false;
                if (a.norm_cut > 0.0) {
                    // y32 = RN32(gn) RN32(c): |y32 - gn c| <= |y32| 2^-22.4 (three roundings)
                    float y32[8];
                    float ymax = 0.f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        y32[i] = __fmul_rn(float(gn[i]), c32);
                        ymax = fmaxf(ymax, fabsf(y32[i]));
                    }
                    const float M = __fadd_rn(__fmul_rn(ymax, 0x1p-21f), 0x1p-40f);
                    double p[8];
                    if (ymax < 64.f && e8_screen(y32, M, p)) {
                        const bool half = p[0] != rint(p[0]);
                        bool in = true;
                        double nrm = 0.0;   // exact: sums of squares of small half-integers
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            in &= half ? (p[i] >= -2.5 && p[i] <= 3.5) : (p[i] >= -3.0 && p[i] <= 3.0);
                            nrm = d_add(nrm, d_mul(p[i], p[i]));
                        }
                        if (in && nrm < a.norm_cut) {
                            double c[8];
                            // grid coordinates are +0.0, never -0.0
#pragma unroll
                            for (int i = 0; i < 8; ++i) c[i] = d_add(p[i], 0.0) / a.scale;
                            store_rec(a, v, c, s);
                            done = true;
                        }
                    }
                }
                pending = !done;
            }
        }
        append(a.list1, a.cnt + 0, pending, unsigned(v));
    }
}

constexpr int kTile = 1024;          // codewords per shared-memory tile (32 KB)
constexpr int kQT = 2;               // vectors per thread
constexpr int kSearchThreads = 256;

// Pass 2.  Persistent CTAs walk list 1 in batches of 512 vectors; every
// batch streams the whole codebook through shared memory.
template <typename TIn>
__global__ void __launch_bounds__(kSearchThreads) qe8_search_kernel(QE8Args a) {
    __shared__ __align__(16) float tile[kTile * 8];
    const unsigned n = *reinterpret_cast<volatile unsigned *>(a.cnt + 0);
    const float cbmax2 = __uint_as_float(*reinterpret_cast<volatile unsigned *>(a.cnt + 3));
    const int tid = threadIdx.x;
    const unsigned tile0 = unsigned(__cvta_generic_to_shared(tile));
    constexpr int64_t kBatch = int64_t(kSearchThreads) * kQT;
    for (int64_t b0 = int64_t(blockIdx.x) * kBatch; b0 < n; b0 += int64_t(gridDim.x) * kBatch) {
        u64 y[kQT][4];
        float d1[kQT], d2[kQT], marg[kQT];
        int i1[kQT];
        bool valid[kQT];
        unsigned vid[kQT];
#pragma unroll
        for (int q = 0; q < kQT; ++q) {
            const int64_t li = b0 + int64_t(q) * kSearchThreads + tid;
            valid[q] = li < n;
            vid[q] = valid[q] ? a.list1[li] : 0u;
            double gn[8], s[8];
            load_gn<TIn>(a, vid[q], gn, s);
            float g[8];
            double g2 = 0.0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                g[i] = float(gn[i]);
                g2 += gn[i] * gn[i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) y[q][i] = pk2(g[2 * i], g[2 * i + 1]);
            marg[q] = float(0x1p-18 * (g2 + double(cbmax2)));
            d1[q] = d2[q] = __int_as_float(0x7f7fffff);
            i1[q] = 0;
        }
        for (int64_t t0 = 0; t0 < a.K; t0 += kTile) {
            const int nt = int(a.K - t0 < kTile ? a.K - t0 : int64_t(kTile));
            __syncthreads();   // the previous tile is consumed
            const float4 *src = reinterpret_cast<const float4 *>(a.cb32 + 8 * t0);
            for (int i = tid; i < 2 * nt; i += kSearchThreads) reinterpret_cast<float4 *>(tile)[i] = __ldg(src + i);
            __syncthreads();
#pragma unroll 4
            for (int j = 0; j < nt; ++j) {
                u64 c01, c23, c45, c67;
                lds2x64(tile0 + 32u * j, c01, c23);
                lds2x64(tile0 + 32u * j + 16u, c45, c67);
                const int jj = int(t0) + j;
#pragma unroll
                for (int q = 0; q < kQT; ++q) {
                    u64 e = sub2(y[q][0], c01);
                    u64 acc = mul2(e, e);
                    e = sub2(y[q][1], c23);
                    acc = fma2(e, e, acc);
                    e = sub2(y[q][2], c45);
                    acc = fma2(e, e, acc);
                    e = sub2(y[q][3], c67);
                    acc = fma2(e, e, acc);
                    float lo, hi;
                    up2(acc, lo, hi);
                    const float d = lo + hi;
                    const bool lt = d < d1[q];
                    d2[q] = fminf(d2[q], fmaxf(d1[q], d));
                    d1[q] = fminf(d1[q], d);
                    i1[q] = lt ? jj : i1[q];
                }
            }
        }
#pragma unroll
        for (int q = 0; q < kQT; ++q) {
            const bool sure = valid[q] && (d2[q] - d1[q] > marg[q]);
            if (sure) {
                double gn[8], s[8], c[8];
                load_gn<TIn>(a, vid[q], gn, s);
#pragma unroll
                for (int i = 0; i < 8; ++i) c[i] = __ldg(a.cb + 8 * int64_t(i1[q]) + i);
                store_rec(a, vid[q], c, s);
            }
            append(a.list2, a.cnt + 1, valid[q] && !sure, vid[q]);
        }
    }
}

// Pass 3: one CTA per listed vector, exact fp64 distances.
template <typename TIn>
__global__ void __launch_bounds__(256) qe8_exact_kernel(QE8Args a) {
    __shared__ double red_d[8];
    __shared__ long long red_j[8];
    const unsigned n = *reinterpret_cast<volatile unsigned *>(a.cnt + 1);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int64_t li = blockIdx.x; li < n; li += gridDim.x) {
        const unsigned v = a.list2[li];
        double gn[8], s[8];
        load_gn<TIn>(a, v, gn, s);
        double best = __longlong_as_double(0x7ff0000000000000ll);
        long long bj = a.K;
        for (int64_t j = tid; j < a.K; j += blockDim.x) {
            double acc = 0.0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const double e = d_sub(gn[i], __ldg(a.cb + 8 * j + i));
                acc = d_add(acc, d_mul(e, e));
            }
            if (acc < best) { best = acc; bj = j; }   // j increases: ties keep the lower index
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const double od = __shfl_xor_sync(0xffffffffu, best, o);
            const long long oj = __shfl_xor_sync(0xffffffffu, bj, o);
            if (od < best || (od == best && oj < bj)) { best = od; bj = oj; }
        }
        if (lane == 0) { red_d[warp] = best; red_j[warp] = bj; }
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < int(blockDim.x) / 32; ++w)
                if (red_d[w] < best || (red_d[w] == best && red_j[w] < bj)) { best = red_d[w]; bj = red_j[w]; }
            if (bj >= a.K) bj = 0;   // unreachable for finite gn (distances are finite)
            double c[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i] = __ldg(a.cb + 8 * bj + i);
            store_rec(a, v, c, s);
        }
        __syncthreads();
    }
}

struct QE8Ws {
    double *rms;
    unsigned *list1, *list2, *cnt;
};

size_t qe8_ws(int64_t size, int64_t group, QE8Ws *w, void *base) {
    const int64_t padded = (size + group - 1) / group * group;
    uq::Carver c(base, ~size_t(0));
    QE8Ws t;
    t.rms = c.take<double>(size_t(padded / group));
    t.list1 = c.take<unsigned>(size_t(padded / 8));
    t.list2 = c.take<unsigned>(size_t(padded / 8));
    t.cnt = c.take<unsigned>(4);
    if (w) *w = t;
    return c.off;
}

template <typename TIn>
int run_qe8(const QE8Args &a, cudaStream_t st) {
    const int64_t sms = uq::num_sms();
    const int g1 = int(std::max<int64_t>(1, std::min<int64_t>((a.nvec + 255) / 256, sms * 16)));
    { uq::ProfScope _p("qe8_classify", st); qe8_classify_kernel<TIn><<<g1, 256, 0, st>>>(a); }
    if (int rc = uq::check_cuda("qe8_classify_kernel launch")) return rc;
    const int64_t batches = (a.nvec + int64_t(kSearchThreads) * kQT - 1) / (int64_t(kSearchThreads) * kQT);
    const int g2 = int(std::max<int64_t>(1, std::min<int64_t>(batches, sms * 4)));
    { uq::ProfScope _p("qe8_search", st); qe8_search_kernel<TIn><<<g2, kSearchThreads, 0, st>>>(a); }
    if (int rc = uq::check_cuda("qe8_search_kernel launch")) return rc;
    const int g3 = int(std::max<int64_t>(1, std::min<int64_t>(a.nvec, sms * 4)));
    { uq::ProfScope _p("qe8_exact", st); qe8_exact_kernel<TIn><<<g3, 256, 0, st>>>(a); }
    return uq::check_cuda("qe8_exact_kernel launch");
}

}  // namespace

extern "C" {

size_t uq_q_e8_workspace_bytes(int64_t size, int64_t group) {
    if (size < 0 || group < 8) return 0;
    return qe8_ws(size, group, nullptr, nullptr);
}

int uq_q_e8(const void *A, int a_dtype, int64_t size, int64_t group, const double *cb, const float *cb32, int64_t K,
            double scale, double norm_cut, double *out, void *workspace, size_t workspace_bytes, void *stream) {
    if (size < 0 || !uq::dtype_size(a_dtype)) return uq::fail(UQ_ERR_INVALID, "uq_q_e8: bad size or dtype");
    if (group < 8 || group % 8 != 0 || group > 8192)
        return uq::fail(UQ_ERR_UNSUPPORTED, "uq_q_e8: group %lld must be a multiple of 8 in [8, 8192]", (long long)group);
    if (K < 1 || K > (int64_t(1) << 31) - 1 || !(scale > 0.0) || !(norm_cut >= 0.0))
        return uq::fail(UQ_ERR_INVALID, "uq_q_e8: bad codebook (K=%lld, scale=%g, norm_cut=%g)", (long long)K, scale,
                        norm_cut);
    const int64_t padded = (size + group - 1) / group * group;
    if (padded / 8 >= (int64_t(1) << 32))
        return uq::fail(UQ_ERR_UNSUPPORTED, "uq_q_e8: %lld elements exceed 2^35", (long long)size);
    if (size == 0) return UQ_OK;
    if (!A || !cb || !cb32 || !out || !workspace) return uq::fail(UQ_ERR_INVALID, "uq_q_e8: null pointer");
    if ((reinterpret_cast<uintptr_t>(cb32) & 15) != 0)
        return uq::fail(UQ_ERR_INVALID, "uq_q_e8: cb32 must be 16-byte aligned");
    QE8Ws w;
    const size_t need = qe8_ws(size, group, &w, workspace);
    if (workspace_bytes < need) return uq::fail(UQ_ERR_WORKSPACE, "uq_q_e8: workspace %zu < %zu", workspace_bytes, need);
    const cudaStream_t st = UQ_STREAM(stream);
    if (cudaMemsetAsync(w.cnt, 0, 4 * sizeof(unsigned), st) != cudaSuccess) return uq::check_cuda("uq_q_e8: clear counters");
    // group scales: sqrt(mean(g^2)) + 1e-12 in numpy's pairwise order
    int rc = uq::e8_quant(A, a_dtype, size, group, 1.0, nullptr, nullptr, w.rms, st);
    if (rc) return rc;
    {
        const int g = int(std::max<int64_t>(1, std::min<int64_t>((K + 255) / 256, int64_t(uq::num_sms()) * 4)));
        uq::ProfScope _p("qe8_cb_norm", st);
        cb_norm_kernel<<<g, 256, 0, st>>>(cb32, K, w.cnt);
    }
    if ((rc = uq::check_cuda("cb_norm_kernel launch"))) return rc;
    QE8Args a{};
    a.A = A; a.size = size; a.group = group; a.nvec = padded / 8; a.rms = w.rms;
    a.cb = cb; a.cb32 = cb32; a.K = K; a.scale = scale; a.norm_cut = norm_cut; a.out = out;
    a.list1 = w.list1; a.list2 = w.list2; a.cnt = w.cnt;
    rc = a_dtype == UQ_F64 ? run_qe8<double>(a, st) : run_qe8<float>(a, st);
    if (rc) return rc;
    // cKDTree.query rejects non-finite points
    unsigned bad = 0;
    if (cudaMemcpyAsync(&bad, w.cnt + 2, sizeof(unsigned), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return uq::check_cuda("uq_q_e8: read status");
    if (bad) return uq::fail(UQ_ERR_INVALID, "'x' must be finite, check for nan or inf values");
    return UQ_OK;
}

}  // extern "C"
