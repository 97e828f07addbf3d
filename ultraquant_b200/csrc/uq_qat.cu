// Differentiable decoder of UltraQuant's QAT step (qat.py:35-59) for sm_100a.
//
//   fwht_torch(x)      qat.py:35-41  butterflies h = 1 .. n/2 in the tensor's
//                                    dtype, then x / sqrt(n)
//   irht_torch(X, n0)  qat.py:43-49  fwht_torch(X) * d, cropped to n0
//   recon_torch(...)   qat.py:51-59  irht_torch(cw[states] * sc_g) / sH
//
// and their gradients as torch autograd forms them: the backward of
// `x / s` is `g / s`, of `a + b, a - b` is `ga + gb, ga - gb` applied in the
// reverse stage order, of `v * d` is `g * d`, of `y / sH` is `g / sH`, and of
// `cw[st] * sc` is the scatter-add of `g * sc` into cw and the per-group sum of
// `g * cw[st]` into sc.  Every per-element step is one correctly rounded
// operation in the tensor's dtype, so the transforms are bit-identical to
// torch on the CPU; the two reductions of the backward accumulate exact fp32
// terms in fp64 (more accurate than torch's fp32 sums, within tolerance).
//
// torch's `x / s` with a Python scalar s = sqrt(n) divides by s rounded to
// the tensor's dtype; for even log2(n) s is a power of two and the division is
// a multiplication by an exact power of two.
//
// Layout: a CTA transforms a tile of 2^NB consecutive elements (NB =
// max(12, b), n = 2^b, 2^(NB-b) rows per tile) held in shared memory with the
// swizzle P(E) = E ^ ((E >> 5) & 31), which keeps every access below free of
// bank conflicts for 4-byte words (8-byte words: two-way at most).  Each of
// the 2^(NB-5) threads keeps 32 elements in registers per pass; pass p keeps
// index bits [p, p+5) in registers.  The tile is filled and (backward) drained
// with thread-consecutive coalesced accesses.
#include <cuda_runtime.h>

#include <algorithm>
#include <stdint.h>

#include "uq_common.cuh"

namespace {

constexpr int VB = 5;           // log2 of the values per thread
constexpr int V = 1 << VB;

__device__ __forceinline__ int swz5(int e) { return e ^ ((e >> 5) & 31); }

template <typename T> struct Ar;
template <> struct Ar<float> {
    static __device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
    static __device__ __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }
    static __device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
    static __device__ __forceinline__ float div(float a, float b) { return __fdiv_rn(a, b); }
};
template <> struct Ar<double> {
    static __device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
    static __device__ __forceinline__ double sub(double a, double b) { return __dsub_rn(a, b); }
    static __device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
    static __device__ __forceinline__ double div(double a, double b) { return __ddiv_rn(a, b); }
};

enum { DIR_FWD = 0, DIR_BWD = 1 };
enum { SRC_DENSE = 0, SRC_RECON = 1 };
enum { DST_DENSE = 0, DST_GRADS = 1 };

struct FwhtArgs {
    int64_t rows;                // rows of the transform (each n = 2^b wide)
    int b;
    // dense source: forward input / backward incoming gradient, (rows, ncols_x)
    const void *x;
    int64_t ld_x, ncols_x;
    // code source (forward) / gradient target (backward): the rotated matrix
    // is rec[f] = cw[states[f]] * sc[f / group], f = row * n + col
    const void *states;
    int states64;
    const float *cw;
    int64_t ncw;
    const float *sc;
    int64_t group;
    int group_shift;             // log2(group) when group is a power of two, else -1
    int64_t ntot;                // rows * n: values of the flat rotated matrix
    const void *signs;           // optional d (n), dtype T
    const void *colscale;        // optional sH (ncols_out forward / ncols_x backward), dtype T
    double s;                    // sqrt(n)
    void *out;
    int64_t ld_out, ncols_out;
    double *gcw, *gsc;           // fp64 gradient accumulators (backward into codes)
    int cw_smem;                 // codebook (and its gradient) staged in shared memory
};

__device__ int g_qat_bad_state = 0;

template <typename T> __device__ __forceinline__ void stage_pair(T &u, T &v) {
    const T a = u, c = v;
    u = Ar<T>::add(a, c);
    v = Ar<T>::sub(a, c);
}

// Butterfly stages of index bits [lo, hi) (all within [p, p+5)) on the 32
// register values x[j] = element(base + (j << p)); ascending for the forward
// transform, descending for its adjoint.
template <typename T, int DIR>
__device__ __forceinline__ void stages32(T (&x)[V], int p, int lo, int hi) {
#pragma unroll
    for (int q = 0; q < VB; ++q) {
        const int lq = DIR == DIR_FWD ? q : VB - 1 - q;
        if (p + lq < lo || p + lq >= hi) continue;
#pragma unroll
        for (int j = 0; j < V; ++j)
            if (!(j & (1 << lq))) stage_pair<T>(x[j], x[j | (1 << lq)]);
    }
}

__device__ __forceinline__ int64_t load_state(const FwhtArgs &a, int64_t f) {
    const int64_t s = a.states64 ? __ldg(static_cast<const long long *>(a.states) + f)
                                 : int64_t(__ldg(static_cast<const int *>(a.states) + f));
    if (s < 0 || s >= a.ncw) {
        atomicExch(&g_qat_bad_state, 1);
        return -1;
    }
    return s;
}

__device__ __forceinline__ int64_t group_of(const FwhtArgs &a, int64_t f) {
    return a.group_shift >= 0 ? (f >> a.group_shift) : f / a.group;
}

template <typename T> struct Vec16;
template <> struct Vec16<float> {
    using type = float4;
    static constexpr int N = 4;
    static __device__ __forceinline__ float4 zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
};
template <> struct Vec16<double> {
    using type = double2;
    static constexpr int N = 2;
    static __device__ __forceinline__ double2 zero() { return make_double2(0.0, 0.0); }
};

// Adjoint of (. / sH), (. * d), (. / s), applied in that order to an incoming
// gradient element of column e.
template <typename T>
__device__ __forceinline__ T bwd_pre(const FwhtArgs &, T v, int e, const T *cs, const T *signs, bool s_pow2,
                                     T s_inv, T s) {
    if (cs) v = Ar<T>::div(v, cs[e]);
    if (signs) v = Ar<T>::mul(v, signs[e]);
    return s_pow2 ? Ar<T>::mul(v, s_inv) : Ar<T>::div(v, s);
}

// Backward into the codes for the 32 consecutive flat elements f0 + j held in
// x[j]: scatter-add x * sc into the codeword gradients (fp64) and per-group
// sums of x * cw[state] into the scale gradients.
template <typename T>
__device__ __forceinline__ void scatter_grads(const FwhtArgs &a, const T (&x)[V], int64_t f0, bool vec_st,
                                              const float *cwp, double *gcwp) {
    double acc = 0.0;
    int64_t g_cur = -1;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        constexpr int HV = V / 2;
        int stv[HV];
        if (vec_st) {
#pragma unroll
            for (int i = 0; i < HV / 4; ++i) {
                const int64_t f = f0 + h * HV + 4 * i;
                int4 q = make_int4(0, 0, 0, 0);
                if (f < a.ntot) q = __ldg(reinterpret_cast<const int4 *>(static_cast<const int *>(a.states) + f));
                stv[4 * i] = q.x; stv[4 * i + 1] = q.y; stv[4 * i + 2] = q.z; stv[4 * i + 3] = q.w;
            }
        }
#pragma unroll
        for (int jj = 0; jj < HV; ++jj) {
            const int j = h * HV + jj;
            const int64_t f = f0 + j;
            if (f >= a.ntot) continue;
            int64_t st;
            if (vec_st) {
                st = stv[jj];
                if (st < 0 || st >= a.ncw) { atomicExch(&g_qat_bad_state, 1); st = -1; }
            } else {
                st = load_state(a, f);
            }
            const int64_t g = group_of(a, f);
            if (st < 0) continue;
            const float gx = float(x[j]);
            atomicAdd(gcwp + st, double(__fmul_rn(gx, __ldg(a.sc + g))));
            if (g != g_cur) {
                if (g_cur >= 0) atomicAdd(a.gsc + g_cur, acc);
                g_cur = g;
                acc = 0.0;
            }
            acc += double(__fmul_rn(gx, cwp[st]));
        }
    }
    if (g_cur >= 0) atomicAdd(a.gsc + g_cur, acc);
}

// ~768 resident threads per SM (80 registers) for the 128- and 256-thread fp32
// tiles, ~384 (168 registers: 32 fp64 values) for fp64.
// BC > 0: the row width 2^BC (>= 4096, one row per tile) is a compile-time
// constant, so every pass, index and branch below folds; BC = 0 reads it from
// the arguments (narrow rows, several per tile).
// MINB > 0 overrides the resident-CTA target: the fp32 gradient kernels with
// the codebook and its fp64 accumulators in shared memory (48 KB) fit 3
// (128 threads) or 2 (256 threads) CTAs per SM anyway, so they take the
// registers that 6 / 3 would leave unused (no spills).
template <typename T, int DIR, int SRC, int DST, int MAXT, int BC, int MINB = 0>
__global__ void __launch_bounds__(MAXT, MINB > 0 ? MINB
                                        : (sizeof(T) == 8 ? (MAXT <= 128 ? 3 : (MAXT <= 256 ? 2 : 1))
                                                          : (MAXT <= 128 ? 6 : (MAXT <= 256 ? 3 : 1))))
fwht_kernel(FwhtArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *tile = reinterpret_cast<T *>(smem_raw);
    using A = Ar<T>;
    const int b = BC ? BC : a.b;
    const int NB = b > 12 ? b : 12;
    const int TILE = 1 << NB;
    const int nthr = 1 << (NB - VB);
    const int tid = threadIdx.x;
    const int nmask = (1 << b) - 1;
    const int64_t n = int64_t(1) << b;
    const int64_t ntiles = (a.rows + (int64_t(1) << (NB - b)) - 1) >> (NB - b);
    const T s = T(a.s);
    const bool s_pow2 = (b & 1) == 0;
    const T s_inv = T(ldexp(1.0, -(b >> 1)));
    const T *signs = static_cast<const T *>(a.signs);
    const T *cs = static_cast<const T *>(a.colscale);
    // small codebooks (L <= 12, the QAT default) live in shared memory after
    // the tile: the gathers and the gradient scatter-add stay on chip
    float *cw_s = reinterpret_cast<float *>(smem_raw + (size_t(sizeof(T)) << NB));
    double *gcw_s = reinterpret_cast<double *>(smem_raw + (size_t(sizeof(T)) << NB) + ((size_t(a.ncw) * 4 + 15) & ~size_t(15)));
    if ((SRC == SRC_RECON || DST == DST_GRADS) && a.cw_smem) {
        for (int i = tid; i < a.ncw; i += nthr) {
            cw_s[i] = __ldg(a.cw + i);
            if (DST == DST_GRADS) gcw_s[i] = 0.0;
        }
        __syncthreads();
    }
    const float *cwp = a.cw_smem ? cw_s : a.cw;
    double *gcwp = a.cw_smem ? gcw_s : a.gcw;
    const bool vec_in = SRC == SRC_RECON
        ? (!a.states64 && b >= 2 && a.group % 4 == 0 && (reinterpret_cast<uintptr_t>(a.states) & 15) == 0)
        : (b >= 2 && a.ncols_x % Vec16<T>::N == 0 && (a.ld_x * int64_t(sizeof(T))) % 16 == 0 &&
           (reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
    const bool vec_st = !a.states64 && b >= 2 && (reinterpret_cast<uintptr_t>(a.states) & 15) == 0;
    const bool vec_out = b >= 2 && a.ncols_out % Vec16<T>::N == 0 && (a.ld_out * int64_t(sizeof(T))) % 16 == 0 &&
                         (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;

    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const int64_t row0 = t << (NB - b);
        // ---- fill: thread-consecutive; 16-byte vectors when aligned, all of a
        //      thread's loads issued before its shared-memory stores ----------
        if (vec_in) {
            if (SRC == SRC_RECON) {
                // in two halves: states (16-byte loads), then all codeword
                // gathers and group scales of the half in flight before use
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    constexpr int HV = V / 2;
                    int stv[HV];
#pragma unroll
                    for (int i = 0; i < HV / 4; ++i) {
                        const int E = (tid + (h * HV / 4 + i) * nthr) * 4;
                        const int64_t f = (t << NB) + E;   // rows of a tile are consecutive in the flat index
                        int4 q = make_int4(0, 0, 0, 0);
                        if (f < a.ntot) q = __ldg(reinterpret_cast<const int4 *>(static_cast<const int *>(a.states) + f));
                        stv[4 * i] = q.x; stv[4 * i + 1] = q.y; stv[4 * i + 2] = q.z; stv[4 * i + 3] = q.w;
                    }
                    float cv[HV];
                    bool bad = false;
#pragma unroll
                    for (int j = 0; j < HV; ++j) {
                        const bool ok = stv[j] >= 0 && stv[j] < a.ncw;
                        bad |= !ok;   // padding past ntot reads state 0, which is valid
                        cv[j] = a.cw_smem ? cwp[ok ? stv[j] : 0] : __ldg(cwp + (ok ? stv[j] : 0));
                        if (!ok) cv[j] = __int_as_float(0x7fc00000);
                    }
                    if (bad) atomicExch(&g_qat_bad_state, 1);
#pragma unroll
                    for (int i = 0; i < HV / 4; ++i) {
                        const int E = (tid + (h * HV / 4 + i) * nthr) * 4;
                        const int64_t f = (t << NB) + E;
                        const bool in = f < a.ntot;
                        const float scv = in ? __ldg(a.sc + group_of(a, f)) : 0.f;   // group % 4 == 0
#pragma unroll
                        for (int j = 0; j < 4; ++j) tile[swz5(E + j)] = in ? T(__fmul_rn(cv[4 * i + j], scv)) : T(0);
                    }
                }
            } else {
                using VT = typename Vec16<T>::type;
                constexpr int VE = Vec16<T>::N;
                VT q[V / VE];
#pragma unroll
                for (int i = 0; i < V / VE; ++i) {
                    const int E = (tid + i * nthr) * VE;
                    const int64_t r = row0 + (E >> b);
                    const int e = E & nmask;
                    q[i] = Vec16<T>::zero();
                    if (r < a.rows && e < a.ncols_x)
                        q[i] = __ldg(reinterpret_cast<const VT *>(static_cast<const T *>(a.x) + r * a.ld_x + e));
                }
#pragma unroll
                for (int i = 0; i < V / VE; ++i) {
                    const int E = (tid + i * nthr) * VE;
                    const int64_t r = row0 + (E >> b);
                    const int e = E & nmask;
                    const bool in = r < a.rows && e < a.ncols_x;
#pragma unroll
                    for (int j = 0; j < VE; ++j) {
                        T v = reinterpret_cast<const T *>(&q[i])[j];
                        if (DIR == DIR_BWD && in) v = bwd_pre<T>(a, v, e + j, cs, signs, s_pow2, s_inv, s);
                        tile[swz5(E + j)] = v;
                    }
                }
            }
        } else {
            for (int E = tid; E < TILE; E += nthr) {
                const int64_t r = row0 + (E >> b);
                const int e = E & nmask;
                T v = T(0);
                if (r < a.rows) {
                    if (SRC == SRC_RECON) {
                        const int64_t f = r * n + e;
                        const int64_t st = load_state(a, f);
                        v = st < 0 ? T(__int_as_float(0x7fc00000))
                                   : T(A::mul(T(cwp[st]), T(__ldg(a.sc + group_of(a, f)))));
                    } else if (e < a.ncols_x) {
                        v = static_cast<const T *>(a.x)[r * a.ld_x + e];
                        if (DIR == DIR_BWD) v = bwd_pre<T>(a, v, e, cs, signs, s_pow2, s_inv, s);
                    }
                }
                tile[swz5(E)] = v;
            }
        }
        __syncthreads();

        T x[V];
        if (DIR == DIR_FWD) {
            int done = 0;
            const int npass = (NB + VB - 1) / VB;
#pragma unroll
            for (int ip = 0; ip < 3; ++ip) {
                if (ip >= npass) break;
                const int p = ip * VB < NB - VB ? ip * VB : NB - VB;
                const int base = (tid & ((1 << p) - 1)) | ((tid >> p) << (p + VB));
#pragma unroll
                for (int j = 0; j < V; ++j) x[j] = tile[swz5(base + (j << p))];
                const int hi = (p + VB < b) ? p + VB : b;
                stages32<T, DIR_FWD>(x, p, done > p ? done : p, hi);
                if (hi > done) done = hi;
                if (p == NB - VB) {
                    // epilogue from registers: base == tid, lanes on consecutive columns
#pragma unroll
                    for (int j = 0; j < V; ++j) {
                        const int E = base + (j << p);
                        const int64_t r = row0 + (E >> b);
                        const int e = E & nmask;
                        if (r >= a.rows || e >= a.ncols_out) continue;
                        T y = s_pow2 ? A::mul(x[j], s_inv) : A::div(x[j], s);
                        if (signs) y = A::mul(y, signs[e]);
                        if (cs) y = A::div(y, cs[e]);
                        static_cast<T *>(a.out)[r * a.ld_out + e] = y;
                    }
                    break;
                }
#pragma unroll
                for (int j = 0; j < V; ++j) tile[swz5(base + (j << p))] = x[j];
                __syncthreads();
            }
        } else {
            int low = b;   // stages of bits >= low are done
            int p = b - VB > 0 ? b - VB : 0;
#pragma unroll
            for (int ip = 0; ip < 4; ++ip) {
                const int base = (tid & ((1 << p) - 1)) | ((tid >> p) << (p + VB));
#pragma unroll
                for (int j = 0; j < V; ++j) x[j] = tile[swz5(base + (j << p))];
                stages32<T, DIR_BWD>(x, p, p, low < p + VB ? low : p + VB);
                low = p;
                if (p == 0) break;
#pragma unroll
                for (int j = 0; j < V; ++j) tile[swz5(base + (j << p))] = x[j];
                __syncthreads();
                p = p - VB > 0 ? p - VB : 0;
            }
            // registers now hold the 32 consecutive elements (tid << 5) + j
            if (DST == DST_GRADS) {
                scatter_grads<T>(a, x, (t << NB) + (tid << VB), vec_st, cwp, gcwp);
            } else {
                const int base = tid << VB;
#pragma unroll
                for (int j = 0; j < V; ++j) tile[swz5(base + j)] = x[j];
                __syncthreads();
                if (vec_out) {
                    using VT = typename Vec16<T>::type;
                    constexpr int VE = Vec16<T>::N;
#pragma unroll
                    for (int i = 0; i < V / VE; ++i) {
                        const int E = (tid + i * nthr) * VE;
                        const int64_t r = row0 + (E >> b);
                        const int e = E & nmask;
                        if (r >= a.rows || e >= a.ncols_out) continue;
                        VT q;
#pragma unroll
                        for (int j = 0; j < VE; ++j) reinterpret_cast<T *>(&q)[j] = tile[swz5(E + j)];
                        *reinterpret_cast<VT *>(static_cast<T *>(a.out) + r * a.ld_out + e) = q;
                    }
                } else {
                    for (int E = tid; E < TILE; E += nthr) {
                        const int64_t r = row0 + (E >> b);
                        const int e = E & nmask;
                        if (r < a.rows && e < a.ncols_out) static_cast<T *>(a.out)[r * a.ld_out + e] = tile[swz5(E)];
                    }
                }
            }
        }
        __syncthreads();   // the tile is refilled for the next tile
    }
    if (DST == DST_GRADS && a.cw_smem) {
        // one global add per codeword and CTA
        for (int i = tid; i < a.ncw; i += nthr)
            if (gcw_s[i] != 0.0) atomicAdd(a.gcw + i, gcw_s[i]);
    }
}


// fp32 rows of n = 2^NB (NB = 12..14), one row per CTA iteration, as
// R = 2^(NB-5) tile rows of 32 columns in shared memory with a row stride of
// 36 floats; R threads hold 32 values each:
//   pass A  thread t: tile row t, elements 32 t + j         (index bits 0..4)
//   pass B  thread t: column t & 31 of rows 32 (t >> 5) + k  (bits 5..9)
//   pass C  thread t: elements t + (k << (NB - 5))           (bits NB-5 .. NB-1)
// Every shared address is a per-thread base plus a compile-time offset, and
// every access is conflict-free: pass A moves 16-byte row chunks (144-byte
// stride: 8 lanes cover the 32 banks), passes B and C put a warp on 32
// consecutive columns of one row.  Pass A is filled straight from global
// memory (or from the codes) and the output leaves from pass C with coalesced
// stores.  Forward only (fwht, irht and recon values); the backward's
// gradient scatter measured faster in fwht_kernel.
constexpr int kRowStride = 36;

template <int DIR, int SRC, int DST, int NB>
__global__ void __launch_bounds__(1 << (NB - 5), NB == 12 ? 6 : (NB == 13 ? 3 : 1))
qat_rows_kernel(FwhtArgs a) {
    static_assert(DIR == DIR_FWD && DST == DST_DENSE, "forward values only");
    using T = float;
    using A = Ar<float>;
    constexpr int R = 1 << (NB - 5), P = NB - 5;
    constexpr int64_t n = int64_t(1) << NB;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float *tq = reinterpret_cast<float *>(smem_raw);
    const int tid = threadIdx.x;
    const float s = float(a.s);
    constexpr bool s_pow2 = (NB & 1) == 0;
    const float s_inv = float(ldexp(1.0, -(NB >> 1)));
    const float *signs = static_cast<const float *>(a.signs);
    const float *cs = static_cast<const float *>(a.colscale);
    // codebooks of up to 4096 entries (L <= 12) are staged after the tile
    float *cw_s = reinterpret_cast<float *>(smem_raw + size_t(R) * kRowStride * 4);
    if (SRC == SRC_RECON && a.cw_smem) {
        for (int i = tid; i < a.ncw; i += R) cw_s[i] = __ldg(a.cw + i);
        __syncthreads();
    }
    const float *cwp = a.cw_smem ? cw_s : a.cw;
    // recon of 4096-wide rows with a staged codebook: sH (ncols_out values) is
    // staged after it (16 KB; measured 20.8 -> 27.1 % of HBM at L = 12).  With
    // the codebook in global memory sH stays there too: the extra shared memory
    // takes L1 from the codebook lookups (measured 16.5 -> 12.6 % at L = 16);
    // wider rows would lose resident CTAs to it.
    const bool cs_smem = SRC == SRC_RECON && NB == 12 && cs && a.cw_smem;
    float *cs_s = reinterpret_cast<float *>(smem_raw + size_t(R) * kRowStride * 4 +
                                            ((size_t(a.ncw) * 4 + 15) & ~size_t(15)));
    if (cs_smem) {
        for (int i = tid; i < a.ncols_out; i += R) cs_s[i] = __ldg(cs + i);
        __syncthreads();
    }
    // bit k: the output column tid + (k << (NB - 5)) takes a negative sign (recon)
    unsigned dneg = 0;
    if (SRC == SRC_RECON && signs) {
#pragma unroll
        for (int k = 0; k < 32; ++k) dneg |= (__ldg(signs + tid + (k << P)) < 0.f ? 1u : 0u) << k;
    }
    const bool vec_st = !a.states64 && (reinterpret_cast<uintptr_t>(a.states) & 15) == 0;
    const bool vec_x = (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (a.ld_x % 4) == 0;
    float *rowA = tq + tid * kRowStride;                                       // pass A
    float *colB = tq + (32 * (tid >> 5)) * kRowStride + (tid & 31);            // pass B, + k * 36
    float *colC = tq + (tid >> 5) * kRowStride + (tid & 31);                   // pass C, + (k << (P-5)) * 36

    for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        float x[V];
        {
            const int e0 = 32 * tid;
            if (SRC == SRC_RECON) {
                const int64_t f0 = row * n + e0;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    int stv[16];
                    if (vec_st) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int4 q = __ldg(reinterpret_cast<const int4 *>(static_cast<const int *>(a.states) + f0 + 16 * h) + i);
                            stv[4 * i] = q.x; stv[4 * i + 1] = q.y; stv[4 * i + 2] = q.z; stv[4 * i + 3] = q.w;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) stv[j] = int(load_state(a, f0 + 16 * h + j));
                    }
                    bool bad = false;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const bool ok = stv[j] >= 0 && stv[j] < a.ncw;
                        bad |= !ok;
                        const float c = a.cw_smem ? cwp[ok ? stv[j] : 0] : __ldg(cwp + (ok ? stv[j] : 0));
                        x[16 * h + j] = ok ? c : __int_as_float(0x7fc00000);
                    }
                    if (bad) atomicExch(&g_qat_bad_state, 1);
                    // one scale when the 16 values share a group (groups of >= 16, aligned)
                    const int64_t g0 = group_of(a, f0 + 16 * h), g1 = group_of(a, f0 + 16 * h + 15);
                    if (g0 == g1) {
                        const float sc = __ldg(a.sc + g0);
#pragma unroll
                        for (int j = 0; j < 16; ++j) x[16 * h + j] = __fmul_rn(x[16 * h + j], sc);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            x[16 * h + j] = __fmul_rn(x[16 * h + j], __ldg(a.sc + group_of(a, f0 + 16 * h + j)));
                    }
                }
            } else {
                const float *src = static_cast<const float *>(a.x) + row * a.ld_x + e0;
                if (vec_x && e0 + 32 <= a.ncols_x) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 q = __ldg(reinterpret_cast<const float4 *>(src) + i);
                        x[4 * i] = q.x; x[4 * i + 1] = q.y; x[4 * i + 2] = q.z; x[4 * i + 3] = q.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) x[j] = e0 + j < a.ncols_x ? __ldg(src + j) : 0.f;
                }
            }
            stages32<T, DIR_FWD>(x, 0, 0, 5);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                *reinterpret_cast<float4 *>(rowA + 4 * i) = make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 32; ++k) x[k] = colB[k * kRowStride];
            stages32<T, DIR_FWD>(x, 5, 5, 10);
#pragma unroll
            for (int k = 0; k < 32; ++k) colB[k * kRowStride] = x[k];
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 32; ++k) x[k] = colC[(k << (P - 5)) * kRowStride];
            stages32<T, DIR_FWD>(x, P, 10, NB);
            float *dst = static_cast<float *>(a.out) + row * a.ld_out;
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                const int e = tid + (k << P);
                if (e >= a.ncols_out) continue;
                float y = s_pow2 ? A::mul(x[k], s_inv) : A::div(x[k], s);
                // recon's d is +-1: the product is a sign flip, read once per CTA
                if (SRC == SRC_RECON) y = ((dneg >> k) & 1u) ? -y : y;
                else if (signs) y = A::mul(y, __ldg(signs + e));
                if (cs) y = A::div(y, cs_smem ? cs_s[e] : __ldg(cs + e));
                dst[e] = y;
            }
        }
        __syncthreads();   // the tile is rewritten for the next row
    }
}

__global__ void grads_to_f32_kernel(const double *g64, int64_t count, float *out) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x)
        out[i] = __double2float_rn(g64[i]);
}

template <int DIR, int SRC, int DST, int NB>
int launch_rows(const FwhtArgs &a, cudaStream_t st, const char *what) {
    const bool codes = SRC == SRC_RECON || DST == DST_GRADS;
    const size_t smem = (size_t(kRowStride) * 4 << (NB - 5)) +
        (codes && a.cw_smem ? ((size_t(a.ncw) * 4 + 15) & ~size_t(15)) + (DST == DST_GRADS ? size_t(a.ncw) * 8 : 0) : 0) +
        (SRC == SRC_RECON && NB == 12 && a.cw_smem && a.colscale ? size_t(a.ncols_out) * 4 : 0);
    auto kern = qat_rows_kernel<DIR, SRC, DST, NB>;
    if (uq::set_smem_attr(reinterpret_cast<const void *>(kern), int(smem)) != cudaSuccess)
        return uq::check_cuda("qat rows: set smem attribute");
    int per_sm = 0;
    if (uq::occupancy_blocks(&per_sm, reinterpret_cast<const void *>(kern), 1 << (NB - 5), smem) != cudaSuccess || per_sm < 1)
        return uq::check_cuda("qat rows: occupancy query");
    const int64_t grid = std::min<int64_t>(a.rows, int64_t(uq::num_sms()) * per_sm);
    if (grid > 0) { uq::ProfScope _p(what, st); kern<<<unsigned(grid), 1 << (NB - 5), smem, st>>>(a); }
    return uq::check_cuda("qat_rows_kernel launch");
}

template <typename T, int DIR, int SRC, int DST>
int launch_fwht(const FwhtArgs &a, cudaStream_t st, const char *what) {
    // forward fp32 rows of 4096..16384: the row-layout kernel (measured faster;
    // the backward's gradient scatter is faster in the tile kernel)
    if constexpr (sizeof(T) == 4 && DIR == DIR_FWD) {
        if (a.b == 12) return launch_rows<DIR, SRC, DST, 12>(a, st, what);
        if (a.b == 13) return launch_rows<DIR, SRC, DST, 13>(a, st, what);
        if (a.b == 14) return launch_rows<DIR, SRC, DST, 14>(a, st, what);
    }
    const int NB = a.b > 12 ? a.b : 12;
    const int nthr = 1 << (NB - VB);
    const bool codes = SRC == SRC_RECON || DST == DST_GRADS;
    const size_t smem = (sizeof(T) << NB) +
        (codes && a.cw_smem ? ((size_t(a.ncw) * 4 + 15) & ~size_t(15)) + (DST == DST_GRADS ? size_t(a.ncw) * 8 : 0) : 0);
    // fp64 tiles stop at n = 16384 (512 threads)
    constexpr int TOP = sizeof(T) == 8 ? 512 : 1024;
    // one-row tiles of 4096 .. 32768 get the width as a compile-time constant
    // (the fp32 forward of 4096 .. 16384 never gets here: qat_rows_kernel)
    constexpr bool ROWS_DONE = sizeof(T) == 4 && DIR == DIR_FWD;
    void (*kern)(FwhtArgs) = fwht_kernel<T, DIR, SRC, DST, 128, 0>;
    if constexpr (!ROWS_DONE) {
        if (a.b == 12) kern = fwht_kernel<T, DIR, SRC, DST, 128, 12>;
        else if (a.b == 13) kern = fwht_kernel<T, DIR, SRC, DST, 256, 13>;
        else if (a.b == 14) kern = fwht_kernel<T, DIR, SRC, DST, 512, 14>;
    }
    if (a.b == 15) kern = fwht_kernel<T, DIR, SRC, DST, TOP, (sizeof(T) == 8 ? 0 : 15)>;
    if constexpr (sizeof(T) == 4 && DST == DST_GRADS) {
        // measured at L = 12: 8.1 -> 8.6 % of HBM (4096 x 4096); with the
        // codebook in global memory (L = 16) 6 CTAs per SM stay faster
        if (a.cw_smem) {
            if (a.b <= 12) kern = a.b == 12 ? fwht_kernel<T, DIR, SRC, DST, 128, 12, 3> : fwht_kernel<T, DIR, SRC, DST, 128, 0, 3>;
            else if (a.b == 13) kern = fwht_kernel<T, DIR, SRC, DST, 256, 13, 2>;
        }
    }
    if (uq::set_smem_attr(reinterpret_cast<const void *>(kern), int(smem)) != cudaSuccess)
        return uq::check_cuda("fwht: set smem attribute");
    int per_sm = 0;
    if (uq::occupancy_blocks(&per_sm, reinterpret_cast<const void *>(kern), nthr, smem) != cudaSuccess || per_sm < 1)
        return uq::check_cuda("fwht: occupancy query");
    const int64_t ntiles = (a.rows + (int64_t(1) << (NB - a.b)) - 1) >> (NB - a.b);
    const int64_t grid = std::min<int64_t>(ntiles, int64_t(uq::num_sms()) * per_sm);
    if (grid > 0) { uq::ProfScope _p(what, st); kern<<<unsigned(grid), nthr, smem, st>>>(a); }
    return uq::check_cuda("fwht_kernel launch");
}

int max_bits(int dtype) { return dtype == UQ_F32 ? 15 : 14; }   // tile <= 128 KB

int set_group(FwhtArgs &a, int64_t group) {
    a.group = group;
    a.group_shift = uq::is_pow2(group) ? uq::ilog2(group) : -1;
    return UQ_OK;
}

}  // namespace

extern "C" {

int uq_fwht(const void *x, int dtype, int64_t rows, int64_t n, int64_t ldx, int64_t ncols_in,
            const void *signs, const void *colscale, int direction, void *out, int64_t ld_out,
            int64_t ncols_out, void *stream) {
    if (rows < 0 || !uq::is_pow2(n) || ncols_in < 0 || ncols_in > n || ldx < ncols_in || ncols_out < 0 ||
        ncols_out > n || ld_out < ncols_out || !uq::dtype_size(dtype) || (direction != 0 && direction != 1))
        return uq::fail(UQ_ERR_INVALID, "uq_fwht: bad arguments (rows=%lld n=%lld ncols_in=%lld ncols_out=%lld dir=%d)",
                        (long long)rows, (long long)n, (long long)ncols_in, (long long)ncols_out, direction);
    if (uq::ilog2(n) > max_bits(dtype))
        return uq::fail(UQ_ERR_UNSUPPORTED, "uq_fwht: n = %lld > %d not built for this dtype", (long long)n,
                        1 << max_bits(dtype));
    if (rows == 0 || ncols_out == 0) return UQ_OK;
    if (!out || (ncols_in > 0 && !x)) return uq::fail(UQ_ERR_INVALID, "uq_fwht: null pointer");
    FwhtArgs a{};
    a.rows = rows; a.b = uq::ilog2(n); a.x = x; a.ld_x = ldx; a.ncols_x = ncols_in;
    a.signs = signs; a.colscale = colscale; a.s = sqrt(double(n));
    a.out = out; a.ld_out = ld_out; a.ncols_out = ncols_out;
    const cudaStream_t st = UQ_STREAM(stream);
    if (direction == 0) {
        if (dtype == UQ_F32) return launch_fwht<float, DIR_FWD, SRC_DENSE, DST_DENSE>(a, st, "fwht");
        return launch_fwht<double, DIR_FWD, SRC_DENSE, DST_DENSE>(a, st, "fwht");
    }
    if (dtype == UQ_F32) return launch_fwht<float, DIR_BWD, SRC_DENSE, DST_DENSE>(a, st, "fwht_bwd");
    return launch_fwht<double, DIR_BWD, SRC_DENSE, DST_DENSE>(a, st, "fwht_bwd");
}

int uq_qat_recon(const void *states, int states64, int64_t nrow, int64_t n, const float *cw, int64_t ncw,
                 const float *sc, int64_t scale_group, const float *signs, const float *sH, int64_t in0,
                 float *out, int64_t ld_out, void *stream) {
    if (nrow < 0 || !uq::is_pow2(n) || ncw < 1 || scale_group < 1 || in0 < 0 || in0 > n || ld_out < in0)
        return uq::fail(UQ_ERR_INVALID, "uq_qat_recon: bad arguments (nrow=%lld n=%lld in0=%lld group=%lld)",
                        (long long)nrow, (long long)n, (long long)in0, (long long)scale_group);
    if (uq::ilog2(n) > max_bits(UQ_F32))
        return uq::fail(UQ_ERR_UNSUPPORTED, "uq_qat_recon: n = %lld > 32768 not built", (long long)n);
    if (nrow == 0 || in0 == 0) return UQ_OK;
    if (!states || !cw || !sc || !signs || !out) return uq::fail(UQ_ERR_INVALID, "uq_qat_recon: null pointer");
    FwhtArgs a{};
    a.rows = nrow; a.b = uq::ilog2(n); a.states = states; a.states64 = states64 ? 1 : 0;
    a.cw = cw; a.ncw = ncw; a.sc = sc; set_group(a, scale_group);
    a.cw_smem = ncw <= 4096 ? 1 : 0;
    a.ntot = nrow * n;
    a.signs = signs; a.colscale = sH; a.s = sqrt(double(n));
    a.out = out; a.ld_out = ld_out; a.ncols_out = in0;
    return launch_fwht<float, DIR_FWD, SRC_RECON, DST_DENSE>(a, UQ_STREAM(stream), "qat_recon");
}

size_t uq_qat_recon_backward_workspace_bytes(int64_t ncw, int64_t ngroups) {
    if (ncw < 0 || ngroups < 0) return 0;
    return uq::align_up(size_t(ncw) * 8, 256) + uq::align_up(size_t(ngroups) * 8, 256);
}

int uq_qat_recon_backward(const float *grad, int64_t ld_grad, const void *states, int states64, int64_t nrow,
                          int64_t n, const float *cw, int64_t ncw, const float *sc, int64_t ngroups,
                          int64_t scale_group, const float *signs, const float *sH, int64_t in0,
                          float *grad_cw, float *grad_sc, void *workspace, size_t workspace_bytes,
                          void *stream) {
    if (nrow < 0 || !uq::is_pow2(n) || ncw < 1 || scale_group < 1 || in0 < 0 || in0 > n || ld_grad < in0 ||
        ngroups < 0)
        return uq::fail(UQ_ERR_INVALID, "uq_qat_recon_backward: bad arguments (nrow=%lld n=%lld in0=%lld)",
                        (long long)nrow, (long long)n, (long long)in0);
    if (uq::ilog2(n) > max_bits(UQ_F32))
        return uq::fail(UQ_ERR_UNSUPPORTED, "uq_qat_recon_backward: n = %lld > 32768 not built", (long long)n);
    if ((nrow * n + scale_group - 1) / scale_group > ngroups)
        return uq::fail(UQ_ERR_INVALID, "uq_qat_recon_backward: %lld scale groups < %lld needed", (long long)ngroups,
                        (long long)((nrow * n + scale_group - 1) / scale_group));
    const size_t need = uq_qat_recon_backward_workspace_bytes(ncw, ngroups);
    if (!workspace || workspace_bytes < need)
        return uq::fail(UQ_ERR_WORKSPACE, "uq_qat_recon_backward: workspace %zu < %zu bytes", workspace_bytes, need);
    if (!grad_cw || !grad_sc || !cw || !sc || !signs || (nrow > 0 && in0 > 0 && (!grad || !states)))
        return uq::fail(UQ_ERR_INVALID, "uq_qat_recon_backward: null pointer");
    const cudaStream_t st = UQ_STREAM(stream);
    uq::Carver c(workspace, workspace_bytes);
    double *gcw = c.take<double>(size_t(ncw));
    double *gsc = c.take<double>(size_t(ngroups));
    if (cudaMemsetAsync(workspace, 0, need, st) != cudaSuccess) return uq::check_cuda("qat backward: memset");
    if (nrow > 0) {
        FwhtArgs a{};
        a.rows = nrow; a.b = uq::ilog2(n); a.x = grad; a.ld_x = ld_grad; a.ncols_x = in0;
        a.states = states; a.states64 = states64 ? 1 : 0; a.cw = cw; a.ncw = ncw; a.sc = sc;
        set_group(a, scale_group);
        a.ntot = nrow * n;
        a.signs = signs; a.colscale = sH; a.s = sqrt(double(n));
        a.gcw = gcw; a.gsc = gsc;
        a.cw_smem = ncw <= 4096 ? 1 : 0;
        const int rc = launch_fwht<float, DIR_BWD, SRC_DENSE, DST_GRADS>(a, st, "qat_recon_bwd");
        if (rc != UQ_OK) return rc;
    }
    {
        uq::ProfScope _p("qat_grads_f32", st);
        const int g1 = int(std::max<int64_t>(1, std::min<int64_t>((ncw + 255) / 256, 1184)));
        grads_to_f32_kernel<<<g1, 256, 0, st>>>(gcw, ncw, grad_cw);
        const int g2 = int(std::max<int64_t>(1, std::min<int64_t>((ngroups + 255) / 256, 1184)));
        if (ngroups > 0) grads_to_f32_kernel<<<g2, 256, 0, st>>>(gsc, ngroups, grad_sc);
    }
    return uq::check_cuda("qat backward: grads_to_f32_kernel launch");
}

}  // extern "C"

namespace uq {
// Reads and clears the sticky "state outside the codebook" flag of the
// decoder kernels (after the caller synchronised).  Returns -1 on a CUDA error.
int qat_take_bad_state() {
    int flag = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&flag, g_qat_bad_state, sizeof(int)) != cudaSuccess) return -1;
    if (flag && cudaMemcpyToSymbol(g_qat_bad_state, &zero, sizeof(int)) != cudaSuccess) return -1;
    return flag;
}
}  // namespace uq
