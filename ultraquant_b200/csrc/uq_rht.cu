// Randomized Hadamard transform along rows (qlab.py:66-98) for sm_100a.
//
// Bit-exactness: the reference runs the Sylvester butterflies in fp64 with
// stage order h = 1, 2, 4, ..., n/2.  Every output is the same sequence of
// correctly rounded adds / subtracts whatever the data layout, so the kernel
// only has to keep the stage order.  Scaling divides by sqrt(n) (forward;
// a multiplication by 2^(-b/2) for even b, else Markstein's correction of
// x * RN(1/sqrt(n)), both correctly rounded) and by n (inverse) exactly like
// numpy.
//
// Layout: a CTA owns a tile of 2^NB consecutive elements (NB = max(12, b),
// n = 2^b; one tile holds 2^(NB-b) rows).  The tile lives in shared memory as
// fp64 with the XOR swizzle P(E) = E ^ ((E >> 4) & 15) on the element index,
// which makes every access pattern below bank-conflict free.  Each of the
// 2^(NB-4) threads holds 16 elements in registers per pass; pass p keeps the
// index bits [p, p+4) in registers and runs the stages of those bits.  The
// final pass (p = NB-4) has consecutive threads on consecutive elements, so
// the global store is coalesced; the load is coalesced the same way.
//
// n = 32768 (fp64 row = 256 KB, above one CTA's shared memory): a cluster of
// two CTAs holds one row, a half each.  Index bits [0, 14) are local to a
// half and run as above; the last stage (h = 16384) pairs element i of the
// first half with element i of the second, which each CTA reads from its
// partner's shared memory (distributed shared memory, plain loads).
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>
#include <stdint.h>

#include "uq_common.cuh"
#include "uq_tma.cuh"

namespace {

constexpr int kTileBits = 14;  // n <= 16384 doubles = 128 KB of shared memory per CTA
constexpr int kMaxBits = 15;   // n = 32768: a row split over a 2-CTA cluster

__device__ __forceinline__ int swz(int e) { return e ^ ((e >> 4) & 15); }

enum { MODE_FWD = 0, MODE_INV = 1 };

// Loads an input element as fp64 (float32 inputs widen exactly).
template <typename T> __device__ __forceinline__ double ld_as_f64(const T *p) { return double(__ldg(p)); }

struct RhtArgs {
    const void *in;
    int64_t rows, n0, ld_in;     // input rows, valid columns, row stride
    int b;                       // log2(n)
    const double *signs;         // n
    const double *colscale;      // optional: fwd multiplies A = in * colscale (n0); inv divides
    const double *pre;           // fwd: colscale * signs (n; signs alone when no colscale)
                                 // inv: colscale * signs (n0), used when colscale is set
    void *out;
    int64_t ld_out, ncols_out;   // output row stride, columns written (< n crops)
    double sqrt_n, n_d;
    double inv_sqrt_n;           // RN(1 / sqrt_n), host IEEE division
    // optional error statistics for the inverse of the importance pipeline:
    // A = rn(W * colscale) recomputed from W, partial sums per CTA.
    const void *ref_w;           // W (rows, n0) with stride ld_w, dtype = ref_dtype
    int64_t ld_w;
    int ref_dtype;
    double *err_partial;         // [gridDim.x * 2]
};

// x / sqrt(n), correctly rounded, for odd log2(n) (the reference divides by
// np.sqrt(n)).  Markstein's final correction (P. Markstein, IBM J. Res. Dev.
// 34(1), 1990): with y = RN(1/d) and q0 = RN(x y) within one ulp of x/d, the
// remainder r = x - q0 d is exact as an FMA and RN(q0 + r y) is the correctly
// rounded quotient.  Magnitudes where an intermediate could leave the normal
// range take the IEEE division.
__device__ __forceinline__ double div_sqrt_n(double x, const RhtArgs &a) {
    const double q0 = d_mul(x, a.inv_sqrt_n);
    const double r = __fma_rn(-q0, a.sqrt_n, x);
    const double q = __fma_rn(r, a.inv_sqrt_n, q0);
    const double ax = fabs(x);
    return (ax > 0x1p-960 && ax < 0x1p960) ? q : x / a.sqrt_n;
}

// Applies the butterfly stages of index bits [lo, hi) that lie in [p, p+4)
// to the 16 register values x[j] = element(base + (j << p)).
__device__ __forceinline__ void stages16(double (&x)[16], int p, int lo, int hi) {
#pragma unroll
    for (int lq = 0; lq < 4; ++lq) {      // stage of index bit p + lq, in order
        if (p + lq < lo || p + lq >= hi) continue;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (!(j & (1 << lq))) {
                const int k = j | (1 << lq);
                const double u = x[j], v = x[k];
                x[j] = d_add(u, v);
                x[k] = d_sub(u, v);
            }
        }
    }
}

// Issues the coalesced 16-byte cp.async copies of tile `t` into the chunk-
// swizzled staging layout at `dst` (zero fill past n0 / the last row): chunk c
// (tile order) of thread u = c / CPT lives at (u * CPT) | ((c % CPT) ^ mix(u)).
template <typename TIn, int MODE>
__device__ __forceinline__ void rht_stage(const RhtArgs &a, const TIn *in, int64_t t, int b, int NB, int nthr,
                                          double *dst_tile) {
    constexpr int EPC = 16 / int(sizeof(TIn));
    constexpr int CPT = 16 / EPC;
    const unsigned sbase = unsigned(__cvta_generic_to_shared(dst_tile));
    const int nmask = (1 << b) - 1;
    const int64_t row0 = t << (NB - b);
    const int64_t lim = (MODE == MODE_FWD) ? a.n0 : (int64_t(1) << b);
    for (int c = threadIdx.x; c < nthr * CPT; c += nthr) {
        const int E = c * EPC;
        const int64_t r = row0 + (E >> b);
        const int e = E & nmask;
        const int u = c / CPT, w = c % CPT;
        const int mix = CPT == 8 ? (u & 7) : ((u >> 1) & 3);
        const unsigned dst = sbase + unsigned(((u * CPT) | (w ^ mix)) * 16);
        int valid = 0;
        if (r < a.rows && e < lim) valid = int((lim - e) < EPC ? (lim - e) : EPC);
        const TIn *src = in + (valid ? r * a.ld_in + e : 0);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                     :: "r"(dst), "l"(src), "r"(valid * int(sizeof(TIn))) : "memory");
    }
}

// Persistent CTAs walk the tiles (gridDim.x apart).  Pass 0 keeps index bits
// [0, 4) in registers (16 consecutive elements per thread), intermediate
// passes go through the swizzled shared tile, the last pass (bits
// [NB-4, NB), consecutive threads on consecutive elements) writes straight to
// global memory.  Fast path (rows of >= 16 elements, 16-byte aligned rows):
// the next tile is prefetched with cp.async into the second buffer while the
// current one is transformed.  Forward: x = rn(a * pre[e]) with
// pre = colscale * signs (a sign flip commutes with rounding, so this equals
// (a * colscale) * signs); padding gives 0 * pre[e] = +-0 as numpy.
template <typename TIn, typename TOut, int MODE, int MAXT, int MINB>
__global__ void __launch_bounds__(MAXT, MINB)
rht_tile_kernel(RhtArgs a, int dbuf) {
    extern __shared__ double smem_d[];
    const int b = a.b;
    const int NB = b > 12 ? b : 12;
    const int nthr = 1 << (NB - 4);
    const int tid = threadIdx.x;
    const int nmask = (1 << b) - 1;
    const int64_t ntiles = (a.rows + (int64_t(1) << (NB - b)) - 1) >> (NB - b);
    const TIn *in = static_cast<const TIn *>(a.in);
    // exact power-of-two scalings replace the divisions when possible
    const bool fwd_pow2 = (b & 1) == 0;
    const double fwd_mul = ldexp(1.0, -(b >> 1));
    const double inv_mul = ldexp(1.0, -b);
    const bool staged = b >= 4 && ((a.ld_in * int64_t(sizeof(TIn))) % 16 == 0) &&
                        ((reinterpret_cast<uintptr_t>(in) & 15) == 0);
    constexpr int EPC = 16 / int(sizeof(TIn));
    constexpr int CPT = 16 / EPC;
    const int TILE = 1 << NB;

    int64_t t = blockIdx.x;
    if (staged && t < ntiles) rht_stage<TIn, MODE>(a, in, t, b, NB, nthr, smem_d);
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int k = 0; t < ntiles; t += gridDim.x, ++k) {
        double *tile = smem_d + ((dbuf && (k & 1)) ? TILE : 0);
        const int64_t row0 = t << (NB - b);
        double x[16];
        // ---- pass 0: load (bits [0, 4) in registers) ------------------------
        {
            const int E0 = tid << 4;
            double raw[16];
            if (staged) {
                if (dbuf) {
                    // prefetch the CTA's next tile into the other buffer
                    const int64_t tn = t + gridDim.x;
                    if (tn < ntiles) rht_stage<TIn, MODE>(a, in, tn, b, NB, nthr, smem_d + ((k & 1) ? 0 : TILE));
                } else if (k > 0) {
                    // single buffer: stage this tile now (the buffer was released
                    // by the barrier that ended the previous tile)
                    rht_stage<TIn, MODE>(a, in, t, b, NB, nthr, smem_d);
                }
                asm volatile("cp.async.commit_group;" ::: "memory");
                if (dbuf) asm volatile("cp.async.wait_group 1;" ::: "memory");
                else asm volatile("cp.async.wait_group 0;" ::: "memory");
                __syncthreads();
                const int mix = CPT == 8 ? (tid & 7) : ((tid >> 1) & 3);
                const TIn *stile = reinterpret_cast<const TIn *>(tile);
#pragma unroll
                for (int w = 0; w < CPT; ++w) {
                    const TIn *q = stile + ((tid * CPT) | (w ^ mix)) * EPC;
#pragma unroll
                    for (int i = 0; i < EPC; ++i) raw[w * EPC + i] = double(q[i]);
                }
                __syncthreads();   // the tile is rewritten by the next pass
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int E = E0 + j;
                    int64_t r = row0 + (E >> b);
                    int e = E & nmask;
                    r = r < a.rows ? r : a.rows - 1;
                    if (MODE == MODE_FWD) e = e < a.n0 ? e : int(a.n0 - 1);
                    raw[j] = ld_as_f64(in + r * a.ld_in + e);
                }
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int E = E0 + j;
                const int64_t r = row0 + (E >> b);
                const int e = E & nmask;
                const bool ok = r < a.rows && (MODE != MODE_FWD || e < a.n0);
                const double v = ok ? raw[j] : 0.0;
                x[j] = MODE == MODE_FWD ? d_mul(v, __ldg(a.pre + e)) : d_mul(v, a.sqrt_n);
            }
            stages16(x, 0, 0, b < 4 ? b : 4);
        }
        int done = b < 4 ? b : 4;
        const int last_p = NB - 4;
        // passes p = 4, 8, ..., last_p (the last one may overlap bits already
        // done): registers of the previous layout -> tile -> layout p
        int prev_p = 0;
        for (int p = 4;; p += 4) {
            if (p > last_p) p = last_p;
            {
                const int pb = (tid & ((1 << prev_p) - 1)) | ((tid >> prev_p) << (prev_p + 4));
#pragma unroll
                for (int j = 0; j < 16; ++j) tile[swz(pb + (j << prev_p))] = x[j];
            }
            __syncthreads();
            const int base = (tid & ((1 << p) - 1)) | ((tid >> p) << (p + 4));
#pragma unroll
            for (int j = 0; j < 16; ++j) x[j] = tile[swz(base + (j << p))];
            const int hi = (p + 4 < b) ? p + 4 : b;
            stages16(x, p, done > p ? done : p, hi);
            if (hi > done) done = hi;
            if (p == last_p) {
                // ---- epilogue: scale and store (coalesced: base == tid) ----
                double se = 0.0, sa = 0.0;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int E = base + (j << p);
                    const int64_t r = row0 + (E >> b);
                    const int e = E & nmask;
                    if (r >= a.rows || e >= a.ncols_out) continue;
                    double y;
                    if (MODE == MODE_FWD) {
                        y = fwd_pow2 ? d_mul(x[j], fwd_mul) : div_sqrt_n(x[j], a);
                    } else {
                        // irht: (x / n) * d, x / n exact; optional / colscale
                        const double xs = d_mul(x[j], inv_mul);
                        y = d_mul(xs, __ldg(a.signs + e));
                        if (a.err_partial) {
                            double w = a.ref_dtype == UQ_F32
                                ? double(__ldg(static_cast<const float *>(a.ref_w) + r * a.ld_w + e))
                                : __ldg(static_cast<const double *>(a.ref_w) + r * a.ld_w + e);
                            const double A = d_mul(w, __ldg(a.colscale + e));
                            const double dd = d_sub(A, y);
                            se = d_add(se, d_mul(dd, dd));
                            sa = d_add(sa, d_mul(A, A));
                        }
                        // (xs * d) / cs == xs / (cs * d): a sign flip commutes with rounding
                        if (a.colscale) y = xs / __ldg(a.pre + e);
                    }
                    static_cast<TOut *>(a.out)[r * a.ld_out + e] = TOut(y);
                }
                if (MODE == MODE_INV && a.err_partial) {
                    // deterministic per-tile reduction: warp tree, then one thread
                    __syncthreads();
                    double *red = tile;
                    for (int o = 16; o > 0; o >>= 1) {
                        se = d_add(se, __shfl_xor_sync(0xffffffffu, se, o));
                        sa = d_add(sa, __shfl_xor_sync(0xffffffffu, sa, o));
                    }
                    const int w = tid >> 5, nw = nthr >> 5;
                    if ((tid & 31) == 0) { red[2 * w] = se; red[2 * w + 1] = sa; }
                    __syncthreads();
                    if (tid == 0) {
                        double s0 = 0.0, s1 = 0.0;
                        for (int i = 0; i < nw; ++i) { s0 = d_add(s0, red[2 * i]); s1 = d_add(s1, red[2 * i + 1]); }
                        a.err_partial[2 * t] = s0;
                        a.err_partial[2 * t + 1] = s1;
                    }
                }
                break;
            }
            __syncthreads();
            prev_p = p;
        }
        __syncthreads();   // this tile buffer is refilled two tiles later
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n"
                 "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void cluster_arrive_rel() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acq() {
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// 8-byte store into a cluster peer's shared memory that completes on the
// peer's mbarrier (complete_tx of 8 bytes): no release fence on the writer
__device__ __forceinline__ void st_async_f64(unsigned addr, double v, unsigned mbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];"
                 :: "r"(addr), "l"(__double_as_longlong(v)), "r"(mbar) : "memory");
}

__device__ __forceinline__ double ld_peer_f64(unsigned addr) {
    double v;
    asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(addr) : "memory");
    return v;
}

// One row of n = 2^15 per cluster of two CTAs (1024 threads, 16 values each,
// one 128 KB half-row tile each); clusters walk the rows.  Stages of bits
// [0, 14) as in rht_tile_kernel on each half; stage 14 combines the halves
// through distributed shared memory.  Partial error sums go to
// err_partial[2 * (2 * row + rank)].
template <typename TIn, typename TOut, int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(1024, 1)
rht_split_kernel(RhtArgs a) {
    extern __shared__ double smem_d[];
    constexpr int NB = kTileBits, HALF = 1 << NB, NTHR = 1 << (NB - 4);
    const int tid = threadIdx.x;
    unsigned rank;
    asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    const int64_t col0 = int64_t(rank) * HALF;
    RhtArgs h = a;                         // this CTA's half as a 2^14-wide problem
    h.b = NB;
    h.rows = a.rows;
    const int64_t n0_loc = a.n0 - col0;
    h.n0 = MODE == MODE_FWD ? (n0_loc < 0 ? 0 : (n0_loc > HALF ? HALF : n0_loc)) : HALF;
    const TIn *in = static_cast<const TIn *>(a.in) + col0;
    constexpr int EPC = 16 / int(sizeof(TIn));
    constexpr int CPT = 16 / EPC;
    const bool staged = ((a.ld_in * int64_t(sizeof(TIn))) % 16 == 0) && ((reinterpret_cast<uintptr_t>(in) & 15) == 0);
    const double inv_mul = ldexp(1.0, -(NB + 1));
    const unsigned peer_tile = [&] {
        unsigned r2;
        asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r2)
            : "r"(unsigned(__cvta_generic_to_shared(smem_d))), "r"(rank ^ 1u));
        return r2;
    }();
    const int64_t nclusters = gridDim.x / 2;
    for (int64_t r = blockIdx.x / 2; r < a.rows; r += nclusters) {
        double x[16];
        {
            double raw[16];
            if (staged) {
                rht_stage<TIn, MODE>(h, in, r, NB, NB, NTHR, smem_d);
                asm volatile("cp.async.commit_group;" ::: "memory");
                asm volatile("cp.async.wait_group 0;" ::: "memory");
                __syncthreads();
                const int mix = CPT == 8 ? (tid & 7) : ((tid >> 1) & 3);
                const TIn *stile = reinterpret_cast<const TIn *>(smem_d);
#pragma unroll
                for (int w = 0; w < CPT; ++w) {
                    const TIn *q = stile + ((tid * CPT) | (w ^ mix)) * EPC;
#pragma unroll
                    for (int i = 0; i < EPC; ++i) raw[w * EPC + i] = double(q[i]);
                }
                __syncthreads();
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    int e = (tid << 4) + j;
                    if (MODE == MODE_FWD && e >= h.n0) e = h.n0 > 0 ? int(h.n0 - 1) : 0;
                    raw[j] = (MODE == MODE_FWD && h.n0 == 0) ? 0.0 : ld_as_f64(in + r * a.ld_in + e);
                }
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int e = (tid << 4) + j;
                const double v = (MODE != MODE_FWD || e < h.n0) ? raw[j] : 0.0;
                x[j] = MODE == MODE_FWD ? d_mul(v, __ldg(a.pre + col0 + e)) : d_mul(v, a.sqrt_n);
            }
            stages16(x, 0, 0, 4);
        }
        int done = 4, prev_p = 0, base = 0;
        for (int p = 4;; p += 4) {
            if (p > NB - 4) p = NB - 4;
            const int pb = (tid & ((1 << prev_p) - 1)) | ((tid >> prev_p) << (prev_p + 4));
#pragma unroll
            for (int j = 0; j < 16; ++j) smem_d[swz(pb + (j << prev_p))] = x[j];
            __syncthreads();
            base = (tid & ((1 << p) - 1)) | ((tid >> p) << (p + 4));
#pragma unroll
            for (int j = 0; j < 16; ++j) x[j] = smem_d[swz(base + (j << p))];
            stages16(x, p, done > p ? done : p, NB);
            done = p + 4;
            if (p == NB - 4) break;
            __syncthreads();
            prev_p = p;
        }
        // ---- stage 14 across the cluster: x_lo + x_hi / x_lo - x_hi ---------
        __syncthreads();
#pragma unroll
        for (int j = 0; j < 16; ++j) smem_d[swz(base + (j << (NB - 4)))] = x[j];
        cluster_sync_all();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const double v = ld_peer_f64(peer_tile + unsigned(swz(base + (j << (NB - 4)))) * 8u);
            x[j] = rank == 0 ? d_add(x[j], v) : d_sub(v, x[j]);
        }
        cluster_sync_all();   // the partner has read this tile before it is restaged
        // ---- epilogue (base == tid: coalesced) ------------------------------
        double se = 0.0, sa = 0.0;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int64_t e = col0 + base + (j << (NB - 4));
            if (e >= a.ncols_out) continue;
            double y;
            if (MODE == MODE_FWD) {
                y = div_sqrt_n(x[j], a);
            } else {
                const double xs = d_mul(x[j], inv_mul);
                y = d_mul(xs, __ldg(a.signs + e));
                if (a.err_partial) {
                    double w = a.ref_dtype == UQ_F32
                        ? double(__ldg(static_cast<const float *>(a.ref_w) + r * a.ld_w + e))
                        : __ldg(static_cast<const double *>(a.ref_w) + r * a.ld_w + e);
                    const double A = d_mul(w, __ldg(a.colscale + e));
                    const double dd = d_sub(A, y);
                    se = d_add(se, d_mul(dd, dd));
                    sa = d_add(sa, d_mul(A, A));
                }
                if (a.colscale) y = xs / __ldg(a.pre + e);
            }
            static_cast<TOut *>(a.out)[r * a.ld_out + e] = TOut(y);
        }
        if (MODE == MODE_INV && a.err_partial) {
            double *red = smem_d;   // the tile is free: the partner is done with it
            for (int o = 16; o > 0; o >>= 1) {
                se = d_add(se, __shfl_xor_sync(0xffffffffu, se, o));
                sa = d_add(sa, __shfl_xor_sync(0xffffffffu, sa, o));
            }
            const int w = tid >> 5;
            if ((tid & 31) == 0) { red[2 * w] = se; red[2 * w + 1] = sa; }
            __syncthreads();
            if (tid == 0) {
                double s0 = 0.0, s1 = 0.0;
                for (int i = 0; i < NTHR / 32; ++i) { s0 = d_add(s0, red[2 * i]); s1 = d_add(s1, red[2 * i + 1]); }
                a.err_partial[2 * (2 * r + rank)] = s0;
                a.err_partial[2 * (2 * r + rank) + 1] = s1;
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// TMA form for rows of n = 2^LB = 4096 or 8192, one CTA per row (wider rows:
// rht_halves_kernel below).  The row arrives by tensor-map loads into a
// shared buffer with the 128-byte swizzle (16-byte chunk c of 128-byte line
// r at c ^ (r & 7)), so that pass 0 -- thread t owns the 16 consecutive
// elements 16t .. 16t+15 -- reads it with conflict-free 16-byte loads; the
// CTA's next row is loaded into the second buffer meanwhile.  The result is
// written back to the buffer in the same swizzled line layout and leaves by
// a tensor-map store.  Columns past n0 (padding) and rows past the end are
// zero-filled by the load and clipped by the store.  Every pass layout is a
// compile-time constant.
// ---------------------------------------------------------------------------
__device__ int g_rht_timeout = 0;

using namespace uq::tma;

__device__ __forceinline__ void rmb_wait(unsigned addr, unsigned parity, bool &fail) {
    mbar_wait_bounded(addr, parity, fail, &g_rht_timeout);
}
__device__ __forceinline__ double flip_if(double v, unsigned neg) {
    return __longlong_as_double(__double_as_longlong(v) ^ (static_cast<long long>(neg) << 63));
}

template <typename TIn, typename TOut, int MODE, int LB, bool COLS>
__global__ void __launch_bounds__(1 << (LB - 4), LB == 12 ? 3 : 1)
rht_tma_kernel(const __grid_constant__ CUtensorMap tin, const __grid_constant__ CUtensorMap tout, RhtArgs a) {
    static_assert(LB == 12 || LB == 13, "rows of 4096 or 8192");
    constexpr int NT = 1 << (LB - 4);
    constexpr int HALF = 1 << LB;                  // elements per row
    constexpr int BUFB = HALF * 8;                 // one buffer: the fp64 tile
    constexpr int NBOX = HALF / 4096;              // tensor-map boxes of 4096 elements
    constexpr int B = LB;                          // log2(n)
    // loads move 4096-element boxes, stores 2048-element boxes
    constexpr int OBOX = 2048, NOBOX = HALF / OBOX;
    constexpr int INB = 4096 * int(sizeof(TIn)), OUTB = OBOX * int(sizeof(TOut));
    extern __shared__ __align__(1024) unsigned char smem_raw_r[];
    __shared__ __align__(8) unsigned long long full[2];
    __shared__ double red[2 * (NT / 32)];
    const int tid = threadIdx.x;
    // the swizzled tensor-map buffers start on a 1024-byte boundary
    unsigned char *smem_r = smem_raw_r + ((1024u - (unsigned(__cvta_generic_to_shared(smem_raw_r)) & 1023u)) & 1023u);
    const unsigned sbase = unsigned(__cvta_generic_to_shared(smem_r));
    const unsigned bar0 = unsigned(__cvta_generic_to_shared(&full[0]));
    const int64_t nctas = gridDim.x;
    const int64_t first = blockIdx.x;
    constexpr int CH_IN = 4096 / (128 / int(sizeof(TIn)));     // 128-byte lines per input box
    constexpr int CH_OUT = OBOX / (128 / int(sizeof(TOut)));
    // Register j holds column tid + (j << (LB - 4)) after the last pass, except
    // for rows of 8192 (LB = 13): their last index bit (12) is done with lane
    // shuffles instead of a third transpose through the tile.  The pass over
    // bits 8..11 reads with lane bit 4 on element bit 12, so register j then
    // holds element (tid & 15) | ((tid >> 5) & 15) << 4 | j << 8 |
    // ((tid >> 4) & 1) << 12.
    constexpr bool SHFL12 = LB == 13;
    auto elem12 = [&](int j) -> int {
        return (tid & 15) | (((tid >> 5) & 15) << 4) | (j << 8) | (((tid >> 4) & 1) << 12);
    };
    // column of register j's output, which is also its index in the store
    // buffer (boxes of 2048 columns)
    auto out_col = [&](int j) -> int {
        if (SHFL12) return elem12(j);
        return tid + (j << (LB - 4));
    };

    if (tid == 0) {
        mbar_init(bar0, 1);
        mbar_init(bar0 + 8, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (tid == 0 && first < a.rows) {
        mbar_arrive_expect_tx(bar0, NBOX * INB);
#pragma unroll
        for (int bx = 0; bx < NBOX; ++bx)
            load3d(sbase + bx * INB, &tin, 0, bx * CH_IN, int(first), bar0);
    }
    // per-thread constants: pass-0 columns 16 tid + j, last-pass columns tid + (j << (LB - 4))
    double pre_r[COLS && MODE == MODE_FWD ? 16 : 1];
    unsigned mask0 = 0, maskL = 0;
    if (MODE == MODE_FWD) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int64_t e = 16 * tid + j;
            if (COLS) pre_r[j] = __ldg(a.pre + e);
            else mask0 |= (__ldg(a.signs + e) < 0.0 ? 1u : 0u) << j;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) maskL |= (__ldg(a.signs + out_col(j)) < 0.0 ? 1u : 0u) << j;
    }
    const double inv_mul = ldexp(1.0, -B);
    const double fwd_mul = ldexp(1.0, -(B >> 1));
    bool fail = false;

    int k = 0;
    for (int64_t r = first; r < a.rows; r += nctas, ++k) {
        const unsigned buf = sbase + unsigned((k & 1) * BUFB);
        double *tile = reinterpret_cast<double *>(smem_r + (k & 1) * BUFB);
        rmb_wait(bar0 + 8u * unsigned(k & 1), unsigned((k >> 1) & 1), fail);
        double x[16];
        // ---- pass 0: 16 consecutive elements from the swizzled lines ----------
        if (sizeof(TIn) == 8) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const double2 v = lds128d(buf + unsigned(tid * 128 + ((c ^ (tid & 7)) << 4)));
                x[2 * c] = v.x;
                x[2 * c + 1] = v.y;
            }
        } else {
            const int ln = tid >> 1, h = tid & 1;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float4 v = lds128f(buf + unsigned(ln * 128 + (((4 * h + c) ^ (ln & 7)) << 4)));
                x[4 * c] = v.x; x[4 * c + 1] = v.y; x[4 * c + 2] = v.z; x[4 * c + 3] = v.w;
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (MODE == MODE_FWD) x[j] = COLS ? d_mul(x[j], pre_r[j]) : flip_if(x[j], (mask0 >> j) & 1u);
            else x[j] = d_mul(x[j], a.sqrt_n);
        }
        stages16(x, 0, 0, 4);
        __syncthreads();   // everyone has its raw values: the buffer becomes the work tile
        // prefetch the CTA's next row into the other buffer (its previous store
        // must have finished reading it)
        if (tid == 0 && r + nctas < a.rows) {
            bulk_wait_read0();
            const unsigned nb = bar0 + 8u * unsigned((k + 1) & 1);
            mbar_arrive_expect_tx(nb, NBOX * INB);
#pragma unroll
            for (int bx = 0; bx < NBOX; ++bx)
                load3d(sbase + unsigned(((k + 1) & 1) * BUFB) + bx * INB, &tin, 0, bx * CH_IN, int(r + nctas), nb);
        }
        // ---- passes 4, 8, ...: transposes through the element-swizzled tile ----
#pragma unroll
        for (int p = 4, prev = 0, done = 4; p - 4 < (SHFL12 ? 8 : LB - 4); p += 4) {
            const int pp = p > LB - 4 ? LB - 4 : p;
            const int pb = (tid & ((1 << prev) - 1)) | ((tid >> prev) << (prev + 4));
#pragma unroll
            for (int j = 0; j < 16; ++j) tile[swz(pb + (j << prev))] = x[j];
            __syncthreads();
            // (SHFL12, bits 8..11: lane bit 4 reads element bit 12; each half
            // warp still covers all banks once)
            const int base = (SHFL12 && pp == 8) ? elem12(0)
                                                 : ((tid & ((1 << pp) - 1)) | ((tid >> pp) << (pp + 4)));
#pragma unroll
            for (int j = 0; j < 16; ++j) x[j] = tile[swz(base + (j << pp))];
            stages16(x, pp, done > pp ? done : pp, SHFL12 ? 12 : LB);
            done = pp + 4;
            prev = pp;
            __syncthreads();
        }
        if constexpr (SHFL12) {
            // stage h = 4096: lanes l and l ^ 16 hold the pair (lower: bit 4 clear)
            const bool upper = (tid >> 4) & 1;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const double o = __shfl_xor_sync(0xffffffffu, x[j], 16);
                x[j] = upper ? d_sub(o, x[j]) : d_add(x[j], o);
            }
        }
        // ---- epilogue: scale, write the swizzled output lines, store ---------
        double se = 0.0, sa = 0.0;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int E = out_col(j);
            const int64_t e = E;
            double y;
            if (MODE == MODE_FWD) {
                y = (B & 1) ? div_sqrt_n(x[j], a) : d_mul(x[j], fwd_mul);
            } else {
                const double xs = d_mul(x[j], inv_mul);
                y = flip_if(xs, (maskL >> j) & 1u);
                if (COLS && e < a.ncols_out) {
                    if (a.err_partial) {
                        const double w = a.ref_dtype == UQ_F32
                            ? double(__ldg(static_cast<const float *>(a.ref_w) + r * a.ld_w + e))
                            : __ldg(static_cast<const double *>(a.ref_w) + r * a.ld_w + e);
                        const double A = d_mul(w, __ldg(a.colscale + e));
                        const double dd = d_sub(A, y);
                        se = d_add(se, d_mul(dd, dd));
                        sa = d_add(sa, d_mul(A, A));
                    }
                    y = xs / __ldg(a.pre + e);
                }
            }
            const unsigned o = buf + swz128<TOut>(E);
            if (sizeof(TOut) == 8) asm volatile("st.shared.f64 [%0], %1;" :: "r"(o), "d"(y) : "memory");
            else asm volatile("st.shared.f32 [%0], %1;" :: "r"(o), "f"(float(y)) : "memory");
        }
        fence_proxy_async();
        if (MODE == MODE_INV && COLS && a.err_partial) {
            for (int o = 16; o > 0; o >>= 1) {
                se = d_add(se, __shfl_xor_sync(0xffffffffu, se, o));
                sa = d_add(sa, __shfl_xor_sync(0xffffffffu, sa, o));
            }
            if ((tid & 31) == 0) { red[2 * (tid >> 5)] = se; red[2 * (tid >> 5) + 1] = sa; }
        }
        __syncthreads();
        if (tid == 0) {
#pragma unroll
            for (int bx = 0; bx < NOBOX; ++bx) store3d(&tout, 0, bx * CH_OUT, int(r), buf + unsigned(bx * OUTB));
            bulk_commit();
            if (MODE == MODE_INV && COLS && a.err_partial) {
                double s0 = 0.0, s1 = 0.0;
                for (int i = 0; i < NT / 32; ++i) { s0 = d_add(s0, red[2 * i]); s1 = d_add(s1, red[2 * i + 1]); }
                a.err_partial[2 * r] = s0;
                a.err_partial[2 * r + 1] = s1;
            }
        }
    }
    if (tid == 0) bulk_wait0();
}

// ---------------------------------------------------------------------------
// n = 16384 in one CTA.  The two 8192-element halves of a row are transformed
// one after the other exactly as the single-CTA rows of 8192 are (index bits
// 0..11 in three passes, bit 12 by lane shuffles), so after each half
// register j of thread t holds element elem12(j) of that half.  The first
// half's 16 values stay in registers while the second is transformed; the
// last stage (index bit 13, pairs (e, e + 8192)) then pairs register j of
// the two halves inside the thread: lower = a + b, upper = a - b, the
// operations of the cluster form, without a cluster or an exchange.
// Halves arrive by tensor-map loads into NBUF rotating 64 KB buffers (half q
// in buffer q % NBUF; the load of half q + NBUF is issued as soon as half q's
// passes are done with the buffer).  Results leave by coalesced stores from
// registers: for each register a half warp writes 16 consecutive columns.
// n = 32768 (CL = 2): a 2-CTA cluster per row, CTA r runs the quarters 2r
// and 2r + 1 (columns r 16384 ..) as above, then the stage of index bit 14
// pairs element e of the two CTAs' 16384: CTA 0 finishes the pairs of its
// sums (quarters 0 and 2), CTA 1 those of its differences (quarters 1 and
// 3), each pushing the other 8192 values into its partner's 64 KB inbox by
// st.async, which completes on the partner's inbox mbarrier.  A split
// cluster barrier per row ("inbox read") keeps the next push behind the
// partner's reads.
// ---------------------------------------------------------------------------
template <typename TIn, typename TOut, int MODE, bool COLS, int NBUF, int CL>
__global__ void __launch_bounds__(512, 1)
rht_halves_kernel(const __grid_constant__ CUtensorMap tin, RhtArgs a) {
    static_assert(CL == 1 || CL == 2, "rows of 16384 (one CTA) or 32768 (two)");
    constexpr int NT = 512, HALF = 8192;
    constexpr int B = CL == 1 ? 14 : 15;                    // log2(n)
    constexpr unsigned INBOX = 8u * HALF;                   // CL = 2: the partner's 8192 values
    constexpr unsigned BUFB = HALF * 8;                     // one fp64 tile
    constexpr int NBOX = HALF / 4096;                       // input boxes of 4096 elements per half
    constexpr unsigned INB = 4096 * unsigned(sizeof(TIn));
    constexpr int EPL = 128 / int(sizeof(TIn));             // elements per 128-byte line
    constexpr int CH_IN = 4096 / EPL, LPH = HALF / EPL;     // lines per box, per half
    extern __shared__ __align__(1024) unsigned char smem_raw_h[];
    __shared__ __align__(8) unsigned long long full[NBUF];
    __shared__ __align__(8) unsigned long long ibar;      // CL = 2: inbox filled
    __shared__ double red[2 * (NT / 32)];
    const int tid = threadIdx.x;
    unsigned rank = 0;
    if (CL > 1) asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    unsigned char *smem_h = smem_raw_h + ((1024u - (unsigned(__cvta_generic_to_shared(smem_raw_h)) & 1023u)) & 1023u);
    const unsigned sbase = unsigned(__cvta_generic_to_shared(smem_h));
    const unsigned bar0 = unsigned(__cvta_generic_to_shared(&full[0]));
    const unsigned ibar0 = unsigned(__cvta_generic_to_shared(&ibar));
    const unsigned inbox = sbase + unsigned(NBUF) * BUFB;   // CL = 2: after the buffers
    const int64_t nctas = gridDim.x / CL, first = blockIdx.x / CL;
    const int col0 = int(rank) * 2 * HALF;                 // this CTA's first column
    // halves q = 0 .. nq-1 of this CTA: row first + (q >> 1) * nctas, half q & 1
    const int64_t nq = first < a.rows ? 2 * ((a.rows - first + nctas - 1) / nctas) : 0;
    auto issue = [&](int64_t q) {   // (one thread) load half q into buffer q % NBUF
        const unsigned bi = unsigned(q % NBUF);
        mbar_arrive_expect_tx(bar0 + 8u * bi, unsigned(NBOX) * INB);
#pragma unroll
        for (int bx = 0; bx < NBOX; ++bx)
            load3d(sbase + bi * BUFB + unsigned(bx) * INB, &tin, 0, col0 / EPL + int(q & 1) * LPH + bx * CH_IN,
                   int(first + (q >> 1) * nctas), bar0 + 8u * bi);
    };
    auto elem12 = [&](int j) -> int {
        return (tid & 15) | (((tid >> 5) & 15) << 4) | (j << 8) | (((tid >> 4) & 1) << 12);
    };
    if (tid == 0) {
        for (int i = 0; i < NBUF; ++i) mbar_init(bar0 + 8u * unsigned(i), 1);
        // CL = 2: the inbox's phase completes on this CTA's arm (arrive +
        // expect_tx) and the partner's INBOX bytes of st.async
        if (CL == 2) mbar_init(ibar0, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (tid == 0)
        for (int64_t q = 0; q < NBUF && q < nq; ++q) issue(q);
    unsigned peer_inbox = 0, peer_ibar = 0;
    if (CL == 2) {
        asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(peer_inbox) : "r"(inbox), "r"(rank ^ 1u));
        asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(peer_ibar) : "r"(ibar0), "r"(rank ^ 1u));
        cluster_arrive_rel();   // opens the first "inbox read" phase (and follows the barrier init)
    }
    // output columns of the sums / differences of register j (last stage)
    auto out_sum = [&](int j) -> int { return (CL == 1 ? 0 : int(rank) * HALF) + elem12(j); };
    auto out_dif = [&](int j) -> int { return (CL == 1 ? HALF : 2 * HALF + int(rank) * HALF) + elem12(j); };
    // sign bits: forward, pass-0 column col0 + h 8192 + 16 tid + j at bit
    // 16 h + j; inverse, output column out_sum(j) at bit j, out_dif(j) at 16 + j
    unsigned smask = 0;
    if (MODE == MODE_FWD) {
        if (!COLS)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    smask |= (__ldg(a.signs + col0 + h * HALF + 16 * tid + j) < 0.0 ? 1u : 0u) << (16 * h + j);
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            smask |= (__ldg(a.signs + out_sum(j)) < 0.0 ? 1u : 0u) << j;
            smask |= (__ldg(a.signs + out_dif(j)) < 0.0 ? 1u : 0u) << (16 + j);
        }
    }
    const double inv_mul = ldexp(1.0, -B);
    const double fwd_mul = ldexp(1.0, -(B >> 1));
    bool fail = false;
    double xa[16];
    for (int64_t q = 0; q < nq; ++q) {
        const int h = int(q & 1);
        const int64_t r = first + (q >> 1) * nctas;
        const unsigned bi = unsigned(q % NBUF);
        const unsigned buf = sbase + bi * BUFB;
        double *tile = reinterpret_cast<double *>(smem_h + bi * BUFB);
        double pre_r[COLS && MODE == MODE_FWD ? 16 : 1];
        if (COLS && MODE == MODE_FWD) {
            // issued before the wait, so their latency overlaps it
#pragma unroll
            for (int j = 0; j < 16; ++j) pre_r[j] = __ldg(a.pre + col0 + h * HALF + 16 * tid + j);
        }
        rmb_wait(bar0 + 8u * bi, unsigned((q / NBUF) & 1), fail);
        double x[16];
        // ---- pass 0: 16 consecutive elements from the swizzled lines ----------
        if (sizeof(TIn) == 8) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const double2 v = lds128d(buf + unsigned(tid * 128 + ((c ^ (tid & 7)) << 4)));
                x[2 * c] = v.x;
                x[2 * c + 1] = v.y;
            }
        } else {
            const int ln = tid >> 1, hl = tid & 1;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float4 v = lds128f(buf + unsigned(ln * 128 + (((4 * hl + c) ^ (ln & 7)) << 4)));
                x[4 * c] = v.x; x[4 * c + 1] = v.y; x[4 * c + 2] = v.z; x[4 * c + 3] = v.w;
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (MODE == MODE_FWD) x[j] = COLS ? d_mul(x[j], pre_r[j]) : flip_if(x[j], (smask >> (16 * h + j)) & 1u);
            else x[j] = d_mul(x[j], a.sqrt_n);
        }
        stages16(x, 0, 0, 4);
        __syncthreads();   // everyone has its raw values: the buffer becomes the work tile
        // ---- pass over bits 4..7 ------------------------------------------------
        {
#pragma unroll
            for (int j = 0; j < 16; ++j) tile[swz((tid << 4) + j)] = x[j];
            __syncthreads();
            const int base = (tid & 15) | ((tid >> 4) << 8);
#pragma unroll
            for (int j = 0; j < 16; ++j) x[j] = tile[swz(base + (j << 4))];
            stages16(x, 4, 4, 12);
            __syncthreads();
        }
        // ---- pass over bits 8..11; lane bit 4 reads element bit 12 ----------------
        {
            const int pb = (tid & 15) | ((tid >> 4) << 8);
#pragma unroll
            for (int j = 0; j < 16; ++j) tile[swz(pb + (j << 4))] = x[j];
            __syncthreads();
            const int base = elem12(0);
#pragma unroll
            for (int j = 0; j < 16; ++j) x[j] = tile[swz(base + (j << 8))];
            stages16(x, 8, 8, 12);
            fence_proxy_async();   // this thread's tile accesses before the next tensor-map load
            __syncthreads();
        }
        // the buffer is free: load the half NBUF ahead into it
        if (tid == 0 && q + NBUF < nq) issue(q + NBUF);
        // stage h = 4096: lanes l and l ^ 16 hold the pair (lower: bit 4 clear)
        {
            const bool upper = (tid >> 4) & 1;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const double o = __shfl_xor_sync(0xffffffffu, x[j], 16);
                x[j] = upper ? d_sub(o, x[j]) : d_add(x[j], o);
            }
        }
        if (h == 0) {
#pragma unroll
            for (int j = 0; j < 16; ++j) xa[j] = x[j];
            continue;
        }
        // ---- stage h = 8192: element e of the first half with e of the second ----
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const double lo = xa[j], hi = x[j];
            xa[j] = d_add(lo, hi);
            x[j] = d_sub(lo, hi);
        }
        if constexpr (CL == 2) {
            // ---- stage h = 16384 with the partner: CTA 0 keeps its sums (quarter
            //      0) and receives CTA 1's (quarter 2); CTA 1 keeps its
            //      differences (quarter 3) and receives CTA 0's (quarter 1) ----
            cluster_wait_acq();   // the partner has read its inbox of the previous row
            if (tid == 0) mbar_arrive_expect_tx(ibar0, INBOX);
#pragma unroll
            for (int j = 0; j < 16; ++j)
                st_async_f64(peer_inbox + 8u * unsigned(elem12(j)), rank ? xa[j] : x[j], peer_ibar);
            rmb_wait(ibar0, unsigned((q >> 1) & 1), fail);   // the partner's values are in the inbox
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const double v = lds64d(inbox + 8u * unsigned(elem12(j)));
                const double own = rank ? x[j] : xa[j];
                const double lo = rank ? v : own, hi = rank ? own : v;
                xa[j] = d_add(lo, hi);
                x[j] = d_sub(lo, hi);
            }
            // inbox read: the partner may push its next row.  The release
            // orders this thread's inbox reads before the partner's next
            // writes (a relaxed arrival measured 5 % faster, but nothing
            // would then keep those reads ahead of it)
            cluster_arrive_rel();
        }
        // ---- epilogue: scale and store (sums at out_sum(j), differences at out_dif(j)) ----
        TOut *orow = static_cast<TOut *>(a.out) + r * a.ld_out;
        double se = 0.0, sa = 0.0;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const double v = hh ? x[j] : xa[j];
                const int64_t e = int64_t(hh ? out_dif(j) : out_sum(j));
                double y;
                if (MODE == MODE_FWD) {
                    y = (B & 1) ? div_sqrt_n(v, a) : d_mul(v, fwd_mul);
                } else {
                    const double xs = d_mul(v, inv_mul);
                    y = flip_if(xs, (smask >> (16 * hh + j)) & 1u);
                    if (COLS && e < a.ncols_out) {
                        if (a.err_partial) {
                            const double w = a.ref_dtype == UQ_F32
                                ? double(__ldg(static_cast<const float *>(a.ref_w) + r * a.ld_w + e))
                                : __ldg(static_cast<const double *>(a.ref_w) + r * a.ld_w + e);
                            const double A = d_mul(w, __ldg(a.colscale + e));
                            const double dd = d_sub(A, y);
                            se = d_add(se, d_mul(dd, dd));
                            sa = d_add(sa, d_mul(A, A));
                        }
                        y = xs / __ldg(a.pre + e);
                    }
                }
                if (MODE == MODE_FWD || e < a.ncols_out) orow[e] = TOut(y);
            }
        }
        if (MODE == MODE_INV && COLS && a.err_partial) {
            for (int o = 16; o > 0; o >>= 1) {
                se = d_add(se, __shfl_xor_sync(0xffffffffu, se, o));
                sa = d_add(sa, __shfl_xor_sync(0xffffffffu, sa, o));
            }
            if ((tid & 31) == 0) { red[2 * (tid >> 5)] = se; red[2 * (tid >> 5) + 1] = sa; }
            __syncthreads();
            if (tid == 0) {
                double s0 = 0.0, s1 = 0.0;
                for (int i = 0; i < NT / 32; ++i) { s0 = d_add(s0, red[2 * i]); s1 = d_add(s1, red[2 * i + 1]); }
                a.err_partial[2 * (CL * r + rank)] = s0;
                a.err_partial[2 * (CL * r + rank) + 1] = s1;
            }
        }
    }
    if (CL == 2) cluster_wait_acq();   // closes the last "inbox read" phase
}

// ---------------------------------------------------------------------------
// Opt-in block-factorised transform for n0 = 28 * P (P = 512 or 1024: the
// ffn_down widths 14336 and 28672 without padding).  No counterpart in the
// reference (it pads to a power of two); the operation order is the one of
// the oracle's rht28_rows / irht28_rows:
//   forward  x = rn(A * colscale) * d; 512/1024-point butterflies in each of
//            the 28 blocks; z_i = sum_k H[i][k] y_k (sequential from +-y_0);
//            out = z * RN(1 / sqrt(N))
//   inverse  w_k = sum_i H[i][k] x_i; block butterflies; y = rn(w * RN(1/sqrt N));
//            out = y * d, or y / (colscale * d)
// H is the Paley type-I Hadamard matrix of order 28 (q = 27); the masks below
// hold its -1 entries (bit k of row i, and bit i of column k).
// One CTA of 512 threads per row, the row in shared memory (the per-block
// swizzle E ^ ((E >> 4) & 15) keeps the butterfly passes and the column reads
// conflict-free).
// ---------------------------------------------------------------------------
__host__ __device__ constexpr unsigned h28_row(int i) {
    constexpr unsigned t[28] = {
    0x0000000u, 0x076e535u, 0x0adea69u, 0x11bf0d3u, 0x38739a5u, 0x5475749u, 0x8c78e93u, 0xc09dd27u, 0xa12be4du, 0x6247c9bu,
    0xdca681du, 0xbd4d02bu, 0x7e1a447u, 0xe7348e1u, 0xeae9151u, 0xf1d2631u, 0x3ba4f03u, 0x57c9a85u, 0x8f93589u, 0x4d03b73u,
    0x9a056f5u, 0x3488df9u, 0x691c39du, 0xd22a3abu, 0xa4c63c7u, 0x49e04efu, 0x935095fu, 0x26b123fu};
    return t[i];
}
__host__ __device__ constexpr unsigned h28_col(int i) {
    constexpr unsigned t[28] = {
    0xffffffeu, 0xf891ac8u, 0xf521592u, 0xee40f24u, 0xc78c64au, 0xab8a896u, 0x738712cu, 0x3f62258u, 0x5ed40b2u, 0x9db8164u,
    0x23593e2u, 0x42b27d4u, 0x81e4bb8u, 0x18c971eu, 0x1512eaeu, 0x0e259ceu, 0xc44b0fcu, 0xa81657au, 0x702ca76u, 0xb27c48cu,
    0x64fa90au, 0xc977206u, 0x92e3c62u, 0x25d5c54u, 0x4b39c38u, 0x961fb10u, 0x2caf6a0u, 0x594edc0u};
    return t[i];
}

struct R28Args {
    const void *in;
    int64_t rows, ld_in;
    int m;                      // P = 2^m
    const double *signs;        // N
    const double *colscale;     // N or null
    void *out;
    int64_t ld_out;
    double c;                   // RN(1 / sqrt(N))
};

// z_i = sum_k (+-) y_k with the signs of row i (or column i when T) of H.
template <bool T>
__device__ __forceinline__ double mix_one(const double (&y)[28], int i) {
    const unsigned mask = T ? h28_col(i) : h28_row(i);
    double acc = (mask & 1u) ? -y[0] : y[0];
#pragma unroll
    for (int k = 1; k < 28; ++k) acc = ((mask >> k) & 1u) ? d_sub(acc, y[k]) : d_add(acc, y[k]);
    return acc;
}

template <typename TIn, typename TOut, int MODE>
__global__ void __launch_bounds__(512, 1) rht28_kernel(R28Args a) {
    extern __shared__ double t28[];
    const int tid = threadIdx.x, m = a.m, P = 1 << m;
    const int N = 28 * P;
    for (int64_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
        // ---- load (forward: scale and sign) ----------------------------------
        const TIn *src = static_cast<const TIn *>(a.in) + r * a.ld_in;
        for (int e = tid; e < N; e += 512) {
            double v = double(__ldg(src + e));
            if (MODE == MODE_FWD) {
                if (a.colscale) v = d_mul(v, __ldg(a.colscale + e));
                v = d_mul(v, __ldg(a.signs + e));
            }
            t28[((e >> m) << m) + swz(e & (P - 1))] = v;
        }
        __syncthreads();
        // ---- column mix (the inverse does it first) ----------------------------
        auto mix_columns = [&](auto Tc, bool to_global) {
            constexpr bool T = decltype(Tc)::value;
            for (int j = tid; j < P; j += 512) {
                const int sj = swz(j);
                double y[28];
#pragma unroll
                for (int k = 0; k < 28; ++k) y[k] = t28[(k << m) + sj];
#pragma unroll
                for (int i = 0; i < 28; ++i) {
                    const double z = mix_one<T>(y, i);
                    if (to_global)
                        static_cast<TOut *>(a.out)[r * a.ld_out + (i << m) + j] = TOut(d_mul(z, a.c));
                    else
                        t28[(i << m) + sj] = z;
                }
            }
        };
        if (MODE == MODE_INV) {
            mix_columns(std::integral_constant<bool, true>{}, false);
            __syncthreads();
        }
        // ---- butterflies inside each of the 28 blocks ---------------------------
        const int tasks = 28 << (m - 4);             // 16 values per task
        int done = 0;
        for (int p = 0;; p += 4) {
            if (p > m - 4) p = m - 4;
            const bool last = p == m - 4;
            for (int u = tid; u < tasks; u += 512) {
                const int k = u >> (m - 4), l = u & ((1 << (m - 4)) - 1);
                const int base = (l & ((1 << p) - 1)) | ((l >> p) << (p + 4));
                double x[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) x[j] = t28[(k << m) + swz(base + (j << p))];
                stages16(x, p, done > p ? done : p, m);
                if (MODE == MODE_INV && last) {
                    // base == l: consecutive tasks write consecutive columns
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int e = (k << m) + base + (j << p);
                        const double xs = d_mul(x[j], a.c);
                        double y;
                        if (a.colscale) y = xs / d_mul(__ldg(a.colscale + e), __ldg(a.signs + e));
                        else y = d_mul(xs, __ldg(a.signs + e));
                        static_cast<TOut *>(a.out)[r * a.ld_out + e] = TOut(y);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) t28[(k << m) + swz(base + (j << p))] = x[j];
                }
            }
            done = p + 4;
            __syncthreads();
            if (last) break;
        }
        if (MODE == MODE_FWD) mix_columns(std::integral_constant<bool, false>{}, true);
        __syncthreads();   // the row buffer is reloaded for the next row
    }
}

template <typename TIn, typename TOut, int MODE>
int launch_rht28(const R28Args &a, cudaStream_t st) {
    auto kern = rht28_kernel<TIn, TOut, MODE>;
    const size_t smem = size_t(28) * (size_t(8) << a.m);
    if (uq::set_smem_attr(reinterpret_cast<const void *>(kern), int(smem)) != cudaSuccess)
        return uq::check_cuda("rht28: set smem attribute");
    const int64_t grid = std::min<int64_t>(a.rows, uq::num_sms());
    if (grid > 0) { uq::ProfScope _p("rht", st); kern<<<unsigned(grid), 512, smem, st>>>(a); }
    return uq::check_cuda("rht28_kernel launch");
}

int rht28_m(int64_t n0) {
    for (int m = 9; m <= 10; ++m)
        if (n0 == 28 * (int64_t(1) << m)) return m;
    return -1;
}

// Fixed-order sum of per-CTA partial pairs -> err[0..1].
__global__ void sum_pairs_kernel(const double *part, int64_t count, double *err) {
    __shared__ double s0[256], s1[256];
    double a = 0.0, c = 0.0;
    for (int64_t i = threadIdx.x; i < count; i += blockDim.x) {
        a = d_add(a, part[2 * i]);
        c = d_add(c, part[2 * i + 1]);
    }
    s0[threadIdx.x] = a;
    s1[threadIdx.x] = c;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) {
            s0[threadIdx.x] = d_add(s0[threadIdx.x], s0[threadIdx.x + w]);
            s1[threadIdx.x] = d_add(s1[threadIdx.x], s1[threadIdx.x + w]);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) { err[0] = s0[0]; err[1] = s1[0]; }
}

// pre[e] = colscale[e] * signs[e] for e < n0, signs[e] beyond (exact products)
__global__ void prescale_kernel(const double *colscale, const double *signs, int64_t n0, int64_t n, double *pre) {
    for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x)
        pre[e] = (colscale && e < n0) ? d_mul(colscale[e], signs[e]) : signs[e];
}

// ---- tensor maps -------------------------------------------------------------
// (rows, ncols) matrix of T with row stride ld, viewed as 128-byte lines:
// dims {elements per line, lines per row, rows}, box = 4096 elements of one row.
template <typename T>
bool make_line_map(CUtensorMap *m, const void *base, int64_t rows, int64_t ncols, int64_t ld, int box_elems) {
    constexpr int EPL = 128 / int(sizeof(T));
    const cuuint64_t dims[3] = {cuuint64_t(EPL), cuuint64_t(ncols / EPL), cuuint64_t(rows)};
    const cuuint64_t strides[2] = {128, cuuint64_t(ld) * sizeof(T)};
    const cuuint32_t box[3] = {cuuint32_t(EPL), cuuint32_t(box_elems / EPL), 1};
    return encode_lines(m, sizeof(T) == 8, 3, base, dims, strides, box);
}

// The TMA form applies to n in {4096, 8192, 16384} with 16-byte aligned
// bases, 16-byte multiple row strides and whole 128-byte lines of valid
// columns (n0 for the input of the forward transform, n0 for the output of
// the inverse).
template <typename TIn, typename TOut>
bool tma_ok(const RhtArgs &a, int64_t ncols_in) {
    if (a.b < 12 || a.b > 15 || a.rows > (int64_t(1) << 31) - 1) return false;
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return al(a.in) && al(a.out) && (a.ld_in * int64_t(sizeof(TIn))) % 16 == 0 &&
           (a.ld_out * int64_t(sizeof(TOut))) % 16 == 0 && ncols_in % (128 / int(sizeof(TIn))) == 0 &&
           a.ncols_out % (128 / int(sizeof(TOut))) == 0 && encode_fn() != nullptr;
}

template <typename TIn, typename TOut, int MODE, int LB, bool COLS>
int launch_tma_v(const CUtensorMap &mi, const CUtensorMap &mo, const RhtArgs &a, cudaStream_t st, int64_t *nparts) {
    auto kern = rht_tma_kernel<TIn, TOut, MODE, LB, COLS>;
    const int nt = 1 << (LB - 4);
    const size_t smem = size_t(2) * (size_t(8) << LB) + 1024;   // two fp64 tiles + alignment slack
    if (uq::set_smem_attr(reinterpret_cast<const void *>(kern), int(smem)) != cudaSuccess)
        return uq::check_cuda("rht tma: set smem attribute");
    int per_sm = 0;
    if (uq::occupancy_blocks(&per_sm, reinterpret_cast<const void *>(kern), nt, smem) != cudaSuccess || per_sm < 1)
        return uq::check_cuda("rht tma: occupancy");
    const int64_t grid = std::min<int64_t>(a.rows, int64_t(per_sm) * uq::num_sms());
    *nparts = a.rows;
    if (grid > 0) {
        uq::ProfScope _p("rht", st);
        kern<<<unsigned(grid), nt, smem, st>>>(mi, mo, a);
    }
    return uq::check_cuda("rht_tma_kernel launch");
}

// Rows of 16384 (CL = 1: three load buffers) or 32768 (CL = 2: a 2-CTA
// cluster per row, two load buffers and the 64 KB inbox).
template <typename TIn, typename TOut, int MODE, bool COLS, int CL>
int launch_tma_halves(const CUtensorMap &mi, const RhtArgs &a, cudaStream_t st, int64_t *nparts) {
    constexpr int NBUF = CL == 1 ? 3 : 2;
    auto kern = rht_halves_kernel<TIn, TOut, MODE, COLS, NBUF, CL>;
    const size_t smem = size_t(NBUF + (CL == 2 ? 1 : 0)) * (size_t(8) << 13) + 1024;   // + alignment slack
    if (uq::set_smem_attr(reinterpret_cast<const void *>(kern), int(smem)) != cudaSuccess)
        return uq::check_cuda("rht halves: set smem attribute");
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(512, 1, 1); cfg.dynamicSmemBytes = smem; cfg.stream = st;
    cfg.attrs = attr; cfg.numAttrs = CL > 1 ? 1 : 0;
    int64_t slots = 0;
    if (CL > 1) {
        cfg.gridDim = dim3(CL, 1, 1);
        int clusters = 0;
        if (uq::occupancy_clusters(&clusters, reinterpret_cast<const void *>(kern), &cfg) != cudaSuccess || clusters < 1)
            return uq::check_cuda("rht halves: cluster occupancy");
        slots = clusters;
    } else {
        int per_sm = 0;
        if (uq::occupancy_blocks(&per_sm, reinterpret_cast<const void *>(kern), 512, smem) != cudaSuccess || per_sm < 1)
            return uq::check_cuda("rht halves: occupancy");
        slots = int64_t(per_sm) * uq::num_sms();
    }
    const int64_t groups = std::min<int64_t>(a.rows, slots);
    cfg.gridDim = dim3(unsigned(groups * CL), 1, 1);
    *nparts = a.rows * CL;   // one error partial per CTA and row
    if (groups > 0) {
        uq::ProfScope _p("rht", st);
        if (cudaLaunchKernelEx(&cfg, kern, mi, a) != cudaSuccess) return uq::check_cuda("rht_halves_kernel launch");
    }
    return uq::check_cuda("rht_halves_kernel launch");
}

template <typename TIn, typename TOut, int MODE, bool COLS>
int launch_tma(const RhtArgs &a, int64_t ncols_in, cudaStream_t st, int64_t *nparts) {
    CUtensorMap mi, mo;
    if (!make_line_map<TIn>(&mi, a.in, a.rows, ncols_in, a.ld_in, 4096) ||
        !make_line_map<TOut>(&mo, a.out, a.rows, a.ncols_out, a.ld_out, 2048))
        return uq::fail(UQ_ERR_CUDA, "rht: tensor map encoding failed");
    // Rows of 4096 and 8192: one CTA per row (rht_tma_kernel; measured on
    // B200, a 512-thread CTA per row of 8192 beats two 4096-element parts on
    // a cluster).  n = 16384 and 32768: each CTA transforms two 8192-element
    // parts in sequence (rht_halves_kernel; one CTA, or a 2-CTA cluster, per
    // row).
    switch (a.b) {
    case 12: return launch_tma_v<TIn, TOut, MODE, 12, COLS>(mi, mo, a, st, nparts);
    case 13: return launch_tma_v<TIn, TOut, MODE, 13, COLS>(mi, mo, a, st, nparts);
    case 14: return launch_tma_halves<TIn, TOut, MODE, COLS, 1>(mi, a, st, nparts);
    default: return launch_tma_halves<TIn, TOut, MODE, COLS, 2>(mi, a, st, nparts);
    }
}

template <typename TIn, typename TOut, int MODE>
int launch_rht_split(const RhtArgs &a, cudaStream_t st) {
    auto kern = rht_split_kernel<TIn, TOut, MODE>;
    const size_t smem = sizeof(double) << kTileBits;
    if (uq::set_smem_attr(reinterpret_cast<const void *>(kern), int(smem)) != cudaSuccess)
        return uq::check_cuda("rht split: set smem attribute");
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2, 1, 1); cfg.blockDim = dim3(1024, 1, 1); cfg.dynamicSmemBytes = smem; cfg.stream = st;
    cfg.attrs = attr; cfg.numAttrs = 1;
    int clusters = 0;
    if (uq::occupancy_clusters(&clusters, reinterpret_cast<const void *>(kern), &cfg) != cudaSuccess || clusters < 1)
        return uq::check_cuda("rht split: cluster occupancy");
    const int64_t ncl = std::min<int64_t>(a.rows, clusters);
    if (ncl > 0) { uq::ProfScope _p("rht", st); kern<<<unsigned(2 * ncl), 1024, smem, st>>>(a); }
    return uq::check_cuda("rht_split_kernel launch");
}

template <typename TIn, typename TOut, int MODE>
int launch_rht(const RhtArgs &a, cudaStream_t st, int64_t *nparts) {
    const int64_t ncols_in = MODE == MODE_FWD ? a.n0 : (int64_t(1) << a.b);
    if (tma_ok<TIn, TOut>(a, ncols_in)) {
        // the colscale form is only used with the pipeline's error statistics or prescale
        if (a.colscale) return launch_tma<TIn, TOut, MODE, true>(a, ncols_in, st, nparts);
        return launch_tma<TIn, TOut, MODE, false>(a, ncols_in, st, nparts);
    }
    {
        const int NB = a.b > 12 ? a.b : 12;
        *nparts = a.b > kTileBits ? 2 * a.rows : (a.rows + (int64_t(1) << (NB - a.b)) - 1) >> (NB - a.b);
    }
    if (a.b > kTileBits) return launch_rht_split<TIn, TOut, MODE>(a, st);
    const int NB = a.b > 12 ? a.b : 12;
    const int nthr = 1 << (NB - 4);
    const int rows_per_tile = 1 << (NB - a.b);
    const int64_t ntiles = (a.rows + rows_per_tile - 1) / rows_per_tile;
    const size_t tile_bytes = sizeof(double) << NB;
    // double-buffer the staged tile when two fit next to each other
    const int dbuf = 2 * tile_bytes <= 160 * 1024 ? 1 : 0;
    const size_t smem = tile_bytes * (dbuf ? 2 : 1);
    // 16 fp64 values per thread; 256-thread tiles (n <= 4096) run 3 CTAs per SM
    auto kern = nthr <= 256 ? rht_tile_kernel<TIn, TOut, MODE, 256, 3>
              : (nthr <= 512 ? rht_tile_kernel<TIn, TOut, MODE, 512, 1> : rht_tile_kernel<TIn, TOut, MODE, 1024, 1>);
    if (uq::set_smem_attr(reinterpret_cast<const void *>(kern), int(smem)) != cudaSuccess)
        return uq::check_cuda("rht: set smem attribute");
    const int per_sm = nthr <= 256 ? 3 : 1;
    const int64_t grid = std::min<int64_t>(ntiles, int64_t(uq::num_sms()) * per_sm);
    if (grid > 0) { uq::ProfScope _p("rht", st); kern<<<unsigned(grid), nthr, smem, st>>>(a, dbuf); }
    return uq::check_cuda("rht_tile_kernel launch");
}

}  // namespace

namespace uq {

int64_t rht_tiles(int64_t rows, int64_t n);

// Forward RHT with optional column pre-scale; output fp64 or fp32.
// pre: colscale * signs (n values) when colscale is given, else nullptr.
int rht_forward(const void *in, int in_dtype, int64_t rows, int64_t n0, int64_t ld_in,
                const double *colscale, const double *pre, const double *signs, void *out, int out_dtype,
                int64_t ld_out, cudaStream_t st) {
    NvtxRange _r("rht_forward");
    RhtArgs a{};
    a.in = in; a.rows = rows; a.n0 = n0; a.ld_in = ld_in;
    const int64_t n = uq_next_pow2(n0);
    a.b = ilog2(n);
    if (colscale && !pre) return fail(UQ_ERR_INVALID, "rht: colscale needs its prescale vector");
    a.signs = signs; a.colscale = colscale; a.pre = colscale ? pre : signs; a.out = out;
    a.ld_out = ld_out; a.ncols_out = n;
    a.sqrt_n = sqrt(double(n)); a.n_d = double(n); a.inv_sqrt_n = 1.0 / a.sqrt_n;
    if (a.b > kMaxBits) return fail(UQ_ERR_UNSUPPORTED, "rht: n = %lld > 32768 not built", (long long)n);
    int64_t nparts = 0;
    if (in_dtype == UQ_F64 && out_dtype == UQ_F64) return launch_rht<double, double, MODE_FWD>(a, st, &nparts);
    if (in_dtype == UQ_F32 && out_dtype == UQ_F64) return launch_rht<float, double, MODE_FWD>(a, st, &nparts);
    if (in_dtype == UQ_F64 && out_dtype == UQ_F32) return launch_rht<double, float, MODE_FWD>(a, st, &nparts);
    if (in_dtype == UQ_F32 && out_dtype == UQ_F32) return launch_rht<float, float, MODE_FWD>(a, st, &nparts);
    return fail(UQ_ERR_INVALID, "rht: bad dtype");
}

// Inverse RHT with optional column post-division and error statistics.
int rht_inverse(const void *in, int in_dtype, int64_t rows, int64_t n, int64_t ld_in,
                int64_t n0, const double *signs, const double *colscale, const double *pre, void *out,
                int out_dtype, int64_t ld_out, const void *ref_w, int ref_dtype,
                int64_t ld_w, double *err_partial, double *err, cudaStream_t st) {
    NvtxRange _r("rht_inverse");
    RhtArgs a{};
    a.in = in; a.rows = rows; a.n0 = n; a.ld_in = ld_in;
    a.b = ilog2(n);
    if (colscale && !pre) return fail(UQ_ERR_INVALID, "irht: colscale needs its prescale vector");
    a.signs = signs; a.colscale = colscale; a.pre = pre; a.out = out;
    a.ld_out = ld_out; a.ncols_out = n0;
    a.sqrt_n = sqrt(double(n)); a.n_d = double(n); a.inv_sqrt_n = 1.0 / a.sqrt_n;
    a.ref_w = ref_w; a.ref_dtype = ref_dtype; a.ld_w = ld_w; a.err_partial = err ? err_partial : nullptr;
    if (a.b > kMaxBits) return fail(UQ_ERR_UNSUPPORTED, "irht: n = %lld > 32768 not built", (long long)n);
    int rc;
    int64_t nparts = 0;
    if (in_dtype == UQ_F64 && out_dtype == UQ_F64) rc = launch_rht<double, double, MODE_INV>(a, st, &nparts);
    else if (in_dtype == UQ_F32 && out_dtype == UQ_F64) rc = launch_rht<float, double, MODE_INV>(a, st, &nparts);
    else if (in_dtype == UQ_F64 && out_dtype == UQ_F32) rc = launch_rht<double, float, MODE_INV>(a, st, &nparts);
    else if (in_dtype == UQ_F32 && out_dtype == UQ_F32) rc = launch_rht<float, float, MODE_INV>(a, st, &nparts);
    else return fail(UQ_ERR_INVALID, "irht: bad dtype");
    if (rc != UQ_OK || !err) return rc;
    { uq::ProfScope _p("sum_pairs", st); sum_pairs_kernel<<<1, 256, 0, st>>>(err_partial, nparts, err); }
    return check_cuda("sum_pairs_kernel launch");
}

int rht_prescale(const double *colscale, const double *signs, int64_t n0, int64_t n, double *pre, cudaStream_t st) {
    const int grid = int(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 1024)));
    { ProfScope _p("prescale", st); prescale_kernel<<<grid, 256, 0, st>>>(colscale, signs, n0, n, pre); }
    return check_cuda("prescale_kernel launch");
}

// Reads and clears the timeout flag of the TMA transform's bounded waits
// (after the caller synchronised); -1 on a CUDA error.
int rht_take_timeout() {
    int flag = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&flag, g_rht_timeout, sizeof(int)) != cudaSuccess) return -1;
    if (flag && cudaMemcpyToSymbol(g_rht_timeout, &zero, sizeof(int)) != cudaSuccess) return -1;
    return flag;
}

// Sets the flag as a timed-out wait would (host-side fault injection).
int rht_set_timeout() {
    const int one = 1;
    return cudaMemcpyToSymbol(g_rht_timeout, &one, sizeof(int)) == cudaSuccess ? 0 : -1;
}

int64_t rht_tiles(int64_t rows, int64_t n) {
    const int b = ilog2(n);
    if (b >= 13) return 4 * rows;   // at most one partial per CTA of a row's cluster
    const int NB = b > 12 ? b : 12;
    return (rows + (1 << (NB - b)) - 1) >> (NB - b);
}

}  // namespace uq

extern "C" {

int uq_rht_rows(const void *A, int a_dtype, int64_t rows, int64_t n0, int64_t lda,
                const double *signs, double *out, void *stream) {
    if (rows < 0 || n0 < 1 || lda < n0 || !uq::dtype_size(a_dtype))
        return uq::fail(UQ_ERR_INVALID, "uq_rht_rows: bad shape (rows=%lld n0=%lld lda=%lld)",
                        (long long)rows, (long long)n0, (long long)lda);
    if (rows == 0) return UQ_OK;
    if (!A || !signs || !out) return uq::fail(UQ_ERR_INVALID, "uq_rht_rows: null pointer");
    const int64_t n = uq_next_pow2(n0);
    return uq::rht_forward(A, a_dtype, rows, n0, lda, nullptr, nullptr, signs, out, UQ_F64, n, UQ_STREAM(stream));
}

int uq_irht_rows(const void *X, int x_dtype, int64_t rows, int64_t n, int64_t ldx, int64_t n0,
                 const double *signs, double *out, void *stream) {
    if (rows < 0 || !uq::is_pow2(n) || ldx < n || n0 < 0 || n0 > n || !uq::dtype_size(x_dtype))
        return uq::fail(UQ_ERR_INVALID, "uq_irht_rows: bad shape (rows=%lld n=%lld n0=%lld)",
                        (long long)rows, (long long)n, (long long)n0);
    if (rows == 0 || n0 == 0) return UQ_OK;
    if (!X || !signs || !out) return uq::fail(UQ_ERR_INVALID, "uq_irht_rows: null pointer");
    return uq::rht_inverse(X, x_dtype, rows, n, ldx, n0, signs, nullptr, nullptr, out, UQ_F64, n0,
                           nullptr, 0, 0, nullptr, nullptr, UQ_STREAM(stream));
}

int uq_rht28_rows(const void *A, int a_dtype, int64_t rows, int64_t n0, int64_t lda, const double *colscale,
                  const double *signs, double *out, void *stream) {
    const int m = rht28_m(n0);
    if (rows < 0 || m < 0 || lda < n0 || !uq::dtype_size(a_dtype))
        return uq::fail(UQ_ERR_INVALID, "uq_rht28_rows: n0 = %lld is not 28 x 512 or 28 x 1024 (rows=%lld lda=%lld)",
                        (long long)n0, (long long)rows, (long long)lda);
    if (rows == 0) return UQ_OK;
    if (!A || !signs || !out) return uq::fail(UQ_ERR_INVALID, "uq_rht28_rows: null pointer");
    R28Args a{};
    a.in = A; a.rows = rows; a.ld_in = lda; a.m = m; a.signs = signs; a.colscale = colscale;
    a.out = out; a.ld_out = n0; a.c = 1.0 / sqrt(double(n0));
    if (a_dtype == UQ_F64) return launch_rht28<double, double, MODE_FWD>(a, UQ_STREAM(stream));
    return launch_rht28<float, double, MODE_FWD>(a, UQ_STREAM(stream));
}

int uq_irht28_rows(const void *X, int x_dtype, int64_t rows, int64_t n0, int64_t ldx, const double *colscale,
                   const double *signs, void *out, int out_dtype, int64_t ld_out, void *stream) {
    const int m = rht28_m(n0);
    if (rows < 0 || m < 0 || ldx < n0 || ld_out < n0 || !uq::dtype_size(x_dtype) || !uq::dtype_size(out_dtype))
        return uq::fail(UQ_ERR_INVALID, "uq_irht28_rows: n0 = %lld is not 28 x 512 or 28 x 1024 (rows=%lld)",
                        (long long)n0, (long long)rows);
    if (rows == 0) return UQ_OK;
    if (!X || !signs || !out) return uq::fail(UQ_ERR_INVALID, "uq_irht28_rows: null pointer");
    R28Args a{};
    a.in = X; a.rows = rows; a.ld_in = ldx; a.m = m; a.signs = signs; a.colscale = colscale;
    a.out = out; a.ld_out = ld_out; a.c = 1.0 / sqrt(double(n0));
    const cudaStream_t st = UQ_STREAM(stream);
    if (x_dtype == UQ_F64 && out_dtype == UQ_F64) return launch_rht28<double, double, MODE_INV>(a, st);
    if (x_dtype == UQ_F64 && out_dtype == UQ_F32) return launch_rht28<double, float, MODE_INV>(a, st);
    if (x_dtype == UQ_F32 && out_dtype == UQ_F64) return launch_rht28<float, double, MODE_INV>(a, st);
    return launch_rht28<float, float, MODE_INV>(a, st);
}

}  // extern "C"
