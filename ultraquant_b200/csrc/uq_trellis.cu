// Bitshift-trellis Viterbi encoder / decoder (trellis.py:14-108, qat.py:11-59)
// for sm_100a.
//
// Recurrence (state s has L bits, a step appends R bits at the bottom):
//   cost_0[s]   = (x_0 - cw[s])^2
//   m_t[q]      = min_k cost_t[k*Q + q],   bp[t+1][q] = first argmin k
//   cost_{t+1}[s] = (x_{t+1} - cw[s])^2 + m_t[s >> R]
// with Q = 2^(L-R), K = 2^R.  Written in terms of m only:
//   m_t[q] = min_k ((x_t - cw[kQ + q])^2 + m_{t-1}[k*Rn + (q >> R)]),  Rn = Q / K.
// Every term is the reference's separate sub / square / add in float32, so
// the min-plus values, and hence the decisions, are bit-exact.
//
// Work split: a thread owns NQ consecutive q (64 = K * NQ trellis states),
// keeps their codewords in registers for the whole sequence and, per step,
//   * reads K * max(NQ/K, 1) values of m_{t-1} from shared memory,
//   * computes its 64 costs with packed f32x2 sub / mul / add,
//   * reduces each q's K candidates with fminf and derives the first-index
//     argmin from the sign bits of f32x2 differences (LOP3 select + funnel
//     shift: no compare / select chains),
//   * writes NQ new m values (16-byte stores) and one 32-bit backpointer word.
// The m array is double buffered in shared memory with an XOR swizzle that
// makes both the write and the read pattern bank-conflict free.
// 2^L / 64 threads cover one sequence: a 512-thread CTA holds several
// sequences for L <= 15; for L = 16 a 2-CTA cluster (2 SMs) shares one
// sequence and reads the other half of m through distributed shared memory.
// Two independent sequence sets are interleaved so that the cluster barrier
// of one set overlaps the arithmetic of the other.
//
// Backpointers go to a global workspace; a second kernel walks them back
// (one thread per sequence) and writes the full L-bit state path.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <type_traits>

#include "uq_common.cuh"
#include "uq_groupsum.cuh"

namespace {

// ---------------------------------------------------------------------------
// Codebook: trellis.py:14-19.  Inverse normal CDF by Wichura's algorithm
// AS 241 (PPND16, Applied Statistics 37(3), 1988), fp64, then float32.
// ---------------------------------------------------------------------------
__device__ double ppnd16(double p) {
    const double q = p - 0.5;
    if (fabs(q) <= 0.425) {
        const double r = 0.180625 - q * q;
        const double num = fma(fma(fma(fma(fma(fma(fma(2.5090809287301226727e+3, r, 3.3430575583588128105e+4), r,
                              6.7265770927008700853e+4), r, 4.5921953931549871457e+4), r,
                              1.3731693765509461125e+4), r, 1.9715909503065514427e+3), r,
                              1.3314166789178437745e+2), r, 3.3871328727963666080e+0);
        const double den = fma(fma(fma(fma(fma(fma(fma(5.2264952788528545610e+3, r, 2.8729085735721942674e+4), r,
                              3.9307895800092710610e+4), r, 2.1213794301586595867e+4), r,
                              5.3941960214247511077e+3), r, 6.8718700749205790830e+2), r,
                              4.2313330701600911252e+1), r, 1.0);
        return q * num / den;
    }
    double r = q < 0 ? p : 1.0 - p;
    r = sqrt(-log(r));
    double val;
    if (r <= 5.0) {
        r -= 1.6;
        const double num = fma(fma(fma(fma(fma(fma(fma(7.74545014278341407640e-4, r, 2.27238449892691845833e-2), r,
                              2.41780725177450611770e-1), r, 1.27045825245236838258e+0), r,
                              3.64784832476320460504e+0), r, 5.76949722146069140550e+0), r,
                              4.63033784615654529590e+0), r, 1.42343711074968357734e+0);
        const double den = fma(fma(fma(fma(fma(fma(fma(1.05075007164441684324e-9, r, 5.47593808499534494600e-4), r,
                              1.51986665636164571966e-2), r, 1.48103976427480074590e-1), r,
                              6.89767334985100004550e-1), r, 1.67638483018380384940e+0), r,
                              2.05319162663775882187e+0), r, 1.0);
        val = num / den;
    } else {
        r -= 5.0;
        const double num = fma(fma(fma(fma(fma(fma(fma(2.01033439929228813265e-7, r, 2.71155556874348757815e-5), r,
                              1.24266094738807843860e-3), r, 2.65321895265761230930e-2), r,
                              2.96560571828504891230e-1), r, 1.78482653991729133580e+0), r,
                              5.46378491116411436990e+0), r, 6.65790464350110377720e+0);
        const double den = fma(fma(fma(fma(fma(fma(fma(2.04426310338993978564e-15, r, 1.42151175831644588870e-7), r,
                              1.84631831751005468180e-5), r, 7.86869131145613259100e-4), r,
                              1.48753612908506148525e-2), r, 1.36929880922735805310e-1), r,
                              5.99832206555887937690e-1), r, 1.0);
        val = num / den;
    }
    return q < 0 ? -val : val;
}

__global__ void codebook_kernel(int L, float *out) {
    const unsigned S = 1u << L;
    for (unsigned s = blockIdx.x * blockDim.x + threadIdx.x; s < S; s += gridDim.x * blockDim.x) {
        unsigned long long h = (unsigned long long)s * 2654435761ull + 0x9E3779B97F4A7C15ull;
        h ^= h >> 29;
        h *= 0xBF58476D1CE4E5B9ull;
        h ^= h >> 32;
        const double u = (double(h & 0xFFFFFFFFull) + 0.5) / 4294967296.0;
        out[s] = float(ppnd16(u));
    }
}

// ---------------------------------------------------------------------------
// Normalisation: trellis.py:69-80 (flat) and :35-42 (per row).
// A CTA stages whole groups in shared memory as float32, reduces the group
// sum of squares in numpy order, and writes sc and xn = g / sc.
// ---------------------------------------------------------------------------
struct NormArgs {
    const void *A;
    int dtype;
    int64_t nrow, T, lda;   // flat mode: nrow = 1, T = ntot, lda = ntot
    int64_t Tp;             // padded row length (flat: padded total)
    int group, tile;        // tile: elements per CTA (multiple of group)
    float *xn, *sc;
};

__device__ __forceinline__ float load_as_f32(const void *A, int dtype, int64_t i) {
    return dtype == UQ_F32 ? __ldg(static_cast<const float *>(A) + i)
                           : float(__ldg(static_cast<const double *>(A) + i));
}

__global__ void normalize_kernel(NormArgs a) {
    extern __shared__ float smf[];
    float *tile = smf;
    const int ng = a.tile / a.group;
    float *ss = tile + a.tile;
    float *scratch = ss + ng;
    const int64_t base = int64_t(blockIdx.x) * a.tile;   // over nrow * Tp
    const int64_t total = a.nrow * a.Tp;
    for (int i = threadIdx.x; i < a.tile; i += blockDim.x) {
        const int64_t gi = base + i;
        float v = 0.f;
        if (gi < total) {
            const int64_t r = gi / a.Tp, c = gi - r * a.Tp;
            if (c < a.T) v = load_as_f32(a.A, a.dtype, r * a.lda + c);
        }
        tile[i] = v;
    }
    __syncthreads();
    tile_group_sumsq<float>(tile, ng, a.group, ss, scratch);
    for (int g = threadIdx.x; g < ng; g += blockDim.x) {
        const int64_t gg = base / a.group + g;
        const float s = __fadd_rn(sqrtf(ss[g] / float(a.group)), 1e-12f);
        ss[g] = s;
        if (gg * a.group < total) a.sc[gg] = s;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < a.tile; i += blockDim.x) {
        const int64_t gi = base + i;
        if (gi < total) a.xn[gi] = tile[i] / ss[i / a.group];
    }
}

// Flat mode, power-of-two groups <= 256: warp per groups, registers only.
template <typename TIn, int G>
__global__ void __launch_bounds__(256) normalize_warp_kernel(NormArgs a) {
    using W = WarpGroup<G>;
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t e_base = warp * W::GPW * int64_t(G);
    const TIn *A = static_cast<const TIn *>(a.A);
    const int64_t ntot = a.T;       // valid elements; a.Tp = padded total
    auto get = [&](int i) -> float {
        const int64_t e = e_base + i;
        return e < ntot ? float(__ldg(A + e)) : 0.f;
    };
    const float ss = warp_group_sumsq<G, float>(get);
    const float sc = __fadd_rn(sqrtf(ss / float(G)), 1e-12f);
    if ((lane % W::LPG) == 0) {
        const int64_t g = e_base / G + lane / W::LPG;
        if (g * G < a.Tp) a.sc[g] = sc;
    }
    for (int vb = 0; vb < W::VPW; vb += 32) {
        const int vv = vb + lane;
        const int gg = (vv < W::VPW ? vv : W::VPW - 1) / W::VPG;
        const float s = __shfl_sync(0xffffffffu, sc, gg * W::LPG);
        if (vv >= W::VPW) continue;
        const int64_t e0 = e_base + 8 * int64_t(vv);
        if (e0 >= a.Tp) continue;
        float x[8];
        if (sizeof(TIn) == 4 && e0 + 8 <= ntot && ((reinterpret_cast<uintptr_t>(A + e0) & 15) == 0)) {
            const float4 *q = reinterpret_cast<const float4 *>(A + e0);
            const float4 t0 = __ldg(q), t1 = __ldg(q + 1);
            x[0] = t0.x; x[1] = t0.y; x[2] = t0.z; x[3] = t0.w; x[4] = t1.x; x[5] = t1.y; x[6] = t1.z; x[7] = t1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = e0 + i < ntot ? float(__ldg(A + e0 + i)) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = x[i] / s;
        if (e0 + 8 <= a.Tp && ((reinterpret_cast<uintptr_t>(a.xn + e0) & 15) == 0)) {
            float4 *q = reinterpret_cast<float4 *>(a.xn + e0);
            q[0] = make_float4(x[0], x[1], x[2], x[3]);
            q[1] = make_float4(x[4], x[5], x[6], x[7]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) if (e0 + i < a.Tp) a.xn[e0 + i] = x[i];
        }
    }
}

template <typename TIn, int G>
int launch_normalize_warp(const NormArgs &a, cudaStream_t st) {
    using W = WarpGroup<G>;
    const int64_t groups = a.Tp / G;
    const int64_t warps = (groups + W::GPW - 1) / W::GPW;
    const int64_t blocks = (warps + 7) / 8;
    if (blocks > 0) { uq::ProfScope _p("normalize", st); normalize_warp_kernel<TIn, G><<<unsigned(blocks), 256, 0, st>>>(a); }
    return uq::check_cuda("normalize_warp_kernel launch");
}

template <typename TIn>
int dispatch_normalize_warp(const NormArgs &a, cudaStream_t st) {
    switch (a.group) {
        case 8: return launch_normalize_warp<TIn, 8>(a, st);
        case 16: return launch_normalize_warp<TIn, 16>(a, st);
        case 32: return launch_normalize_warp<TIn, 32>(a, st);
        case 64: return launch_normalize_warp<TIn, 64>(a, st);
        case 128: return launch_normalize_warp<TIn, 128>(a, st);
        case 256: return launch_normalize_warp<TIn, 256>(a, st);
    }
    return -1;
}

int launch_normalize(NormArgs a, cudaStream_t st) {
    if (a.nrow == 1) {   // flat mode (trellis.py:69-80)
        const int rc = a.dtype == UQ_F32 ? dispatch_normalize_warp<float>(a, st) : dispatch_normalize_warp<double>(a, st);
        if (rc >= 0) return rc;
    }
    int t = a.group;
    while (t < 2048) t += a.group;
    a.tile = t;
    const int ng = a.tile / a.group;
    const size_t smem = sizeof(float) * (size_t(a.tile) + ng + size_t(ng) * 32);
    const int64_t total = a.nrow * a.Tp;
    const int64_t grid = (total + a.tile - 1) / a.tile;
    if (uq::set_smem_attr(reinterpret_cast<const void *>(normalize_kernel), int(smem)) != cudaSuccess)
        return uq::check_cuda("normalize: set smem attribute");
    if (grid > 0) { uq::ProfScope _p("normalize", st); normalize_kernel<<<unsigned(grid), 256, smem, st>>>(a); }
    return uq::check_cuda("normalize_kernel launch");
}

// ---------------------------------------------------------------------------
// Viterbi forward
// ---------------------------------------------------------------------------
constexpr int kThreads = 512;

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
// RN(d * d) for both halves, as a packed FMA with a +0 addend.  ptxas
// contracts a mul.rn.f32x2 whose result feeds an add.rn.f32x2 into a single
// fma.rn.f32x2 -- one rounding where the reference rounds the square and
// then the sum -- even with -fmad=false (observed on sm_100a: m values one
// ulp off, and one path in 65,536 of a 4096 x 4096 tensor changed).  An
// FMA's rounded result cannot be fused any further, and d*d + (+0) rounds
// exactly like d*d (a zero square stays +0).
__device__ __forceinline__ u64 sq2(u64 d) {
    u64 r;
    const u64 zero = 0ull;
    asm("fma.rn.f32x2 %0, %1, %1, %2;" : "=l"(r) : "l"(d), "l"(zero));
    return r;
}
__device__ __forceinline__ u64 add2(u64 a, u64 b) {
    u64 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// min of three float32 values (the 3-input form of min.f32, sm_100): exact,
// so the order of the operands does not matter for non-NaN costs
__device__ __forceinline__ float min3f(float a, float b, float c) {
    float r;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
// bitwise select by the mask word: (m & a) | (~m & b); only bit 31 is used.
__device__ __forceinline__ unsigned sel_bits(unsigned m, unsigned a, unsigned b) {
    unsigned r;
    asm("lop3.b32 %0, %1, %2, %3, 0xCA;" : "=r"(r) : "r"(m), "r"(a), "r"(b));
    return r;
}
// insert the low `len` bits of a into b at bit `pos`
__device__ __forceinline__ unsigned bfi(unsigned a, unsigned b, int pos, int len) {
    unsigned r;
    asm("bfi.b32 %0, %1, %2, %3, %4;" : "=r"(r) : "r"(a), "r"(b), "r"(pos), "r"(len));
    return r;
}
// (word << 1) | (src >> 31)
__device__ __forceinline__ unsigned shift_in_sign(unsigned word, unsigned src) {
    unsigned r;
    asm("shf.l.wrap.b32 %0, %1, %2, 1;" : "=r"(r) : "r"(src), "r"(word));
    return r;
}

__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;\n" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;\n" ::: "memory"); }
__device__ __forceinline__ unsigned cluster_rank() {
    unsigned r;
    asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ unsigned mapa_shared(unsigned addr, unsigned rank) {
    unsigned r;
    asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 lds4(unsigned addr, bool cluster) {
    float4 v;
    if (cluster)
        asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    else
        asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ float lds1(unsigned addr, bool cluster) {
    float v;
    if (cluster) asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    else asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ void sts4(unsigned addr, float a, float b, float c, float d) {
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" :: "r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}
__device__ __forceinline__ void sts4_cluster(unsigned addr, float a, float b, float c, float d) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1,%2,%3,%4};" :: "r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

template <int R> struct Swz;
template <> struct Swz<1> { static constexpr int A = 3, M = 7; };
template <> struct Swz<2> { static constexpr int A = 2, M = 7; };
template <> struct Swz<3> { static constexpr int A = 1, M = 7; };
template <> struct Swz<4> { static constexpr int A = 1, M = 0; };

template <int R> __device__ __forceinline__ unsigned swz_chunk(unsigned c) {
    return c ^ ((c >> Swz<R>::A) & Swz<R>::M);
}

struct VitArgs {
    const float *xn;        // (nseq, T) normalised values
    int64_t seq0, nbatch;   // sequences [seq0, seq0 + nbatch) in this launch
    int T;
    const float *cw;        // 2^L
    uint32_t *bp;           // (nbatch, T-1, TPS)
    int32_t *fin;           // (nbatch)
};

template <int L_, int R_, int CL_> struct VitCfg {
    static constexpr int L = L_, R = R_, CL = CL_;
    static constexpr int K = 1 << R;
    static constexpr int NQ = 64 / K;                    // q per thread (64 states)
    static constexpr int NP = NQ / 2;                    // f32x2 pairs per thread
    static constexpr int NR = NQ >= K ? NQ / K : 1;      // m values read per k
    static constexpr int Q = 1 << (L - R);
    static constexpr int Rn = Q >> R;
    static constexpr int TPS = Q / NQ;                   // threads per sequence
    static constexpr int NSET = (CL == 2 && R >= 2) ? 2 : 1;   // interleaved sets (cluster)
    static constexpr int NBUF = 2;                       // m buffers per set
    // step loop unrolled by two (buffer parities become constants) where that
    // measured faster; R = 1 and 4 spill when unrolled
    static constexpr int UNROLL = R_ == 2 || R_ == 3 ? 2 : 1;
    static constexpr int SPS = CL == 1 ? kThreads / TPS : 1;   // sequences per set per CTA
    // Decision record per q.  R = 2, 3: the raw signs s_k = signbit(m - c_k)
    // for k < K - 1 (F = K - 1 bits; s_k = 0 iff c_k is the minimum m, so the
    // first-index argmin is the lowest clear bit, K - 1 if none).  This saves
    // the tournament's subtree selects, and m takes 3-input mins.  R = 1, 4:
    // the tournament's R-bit index.  A thread's record of one step is BPW
    // 32-bit words; word w holds q-local jq in [w HQ, (w+1) HQ).  R = 1, 4:
    // field at bits F (jq % HQ) .. + F.  R = 2, 3: pair pw = (jq % HQ) / 2 of
    // the word occupies bits 2F pw .. + 2F, s_k of jq at bit 2F pw + 2k +
    // (jq & 1).
    static constexpr bool RAW = R_ == 2 || R_ == 3;
    static constexpr int F = RAW ? K - 1 : R_;
    static constexpr int BPW = (NQ * F + 31) / 32;
    static constexpr int HQ = NQ / BPW;
    static_assert(!RAW || (HQ % 4 == 0 && 4 * F <= 32), "a 4-q chunk fits one word");
    static constexpr int FLOATS = kThreads * NQ;         // floats per (set, buffer) per CTA
    static constexpr int A = Swz<R>::A, M = Swz<R>::M;
    // k-strides (Rn floats per CTA, Rn/2 in a cluster) and slot strides leave
    // the swizzle source bits untouched: addresses are base + constants
    static constexpr int KSTRIDE = CL == 2 ? Rn / 2 : Rn;
    static constexpr bool FAST = (KSTRIDE % (4 << (A + 3))) == 0;
    // cluster mode: the CTA reading a thread's outputs is bit TBIT of v, so
    // half of each CTA's warps write locally and half into the peer
    static constexpr int TBIT = L - R - 7;
    // cluster mode: CTA r's threads produce half r (Q/4 floats, Q bytes) of
    // both CTAs' buffers; the peer's share is staged in a local outbox and
    // moved with one bulk copy per step
    static constexpr unsigned OBYTES = unsigned(Q);
    static constexpr int OFLOATS = CL == 2 ? Q / 4 : 0;
    static_assert(CL == 1 ? TPS <= kThreads : TPS == CL * kThreads, "thread split");
    static_assert(CL == 1 || (TBIT >= 5 && TBIT < 9), "writer target must be warp uniform");
};

// Tournament over K candidate pairs: min pair and R decision words per
// component (bit 31 = "right child wins"; ties keep the left = first index).
template <int R>
__device__ __forceinline__ u64 tourney(const u64 (&c)[1 << R], unsigned (&blo)[R], unsigned (&bhi)[R]) {
    constexpr int K = 1 << R;
    u64 val[K];
#pragma unroll
    for (int k = 0; k < K; ++k) val[k] = c[k];
    // P[j][i]: decision word of the level-(j+1) node on the chosen path of subtree i
    unsigned Plo[R][K], Phi[R][K];
#pragma unroll
    for (int lev = 1; lev <= R; ++lev) {
        const int width = K >> lev;
#pragma unroll
        for (int i = 0; i < width; ++i) {
            const u64 d = sub2(val[2 * i + 1], val[2 * i]);
            float dl, dh;
            up2(d, dl, dh);
            const unsigned wl = __float_as_uint(dl), wh = __float_as_uint(dh);
#pragma unroll
            for (int j = 0; j < lev - 1; ++j) {
                Plo[j][i] = sel_bits(wl, Plo[j][2 * i + 1], Plo[j][2 * i]);
                Phi[j][i] = sel_bits(wh, Phi[j][2 * i + 1], Phi[j][2 * i]);
            }
            Plo[lev - 1][i] = wl;
            Phi[lev - 1][i] = wh;
            float al, ah, bl, bh;
            up2(val[2 * i], al, ah);
            up2(val[2 * i + 1], bl, bh);
            val[i] = pk2(fminf(al, bl), fminf(ah, bh));
        }
    }
#pragma unroll
    for (int j = 0; j < R; ++j) { blo[j] = Plo[j][0]; bhi[j] = Phi[j][0]; }
    return val[0];
}

// ---- mbarrier helpers (cluster exchange) ------------------------------------
__device__ __forceinline__ void mbar_init(unsigned addr, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(addr), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned addr, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(addr), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned addr) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(addr) : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Waits for the phase with the given parity.  Bounded: after limit_ns the
// wait records a timeout in *err and returns true, and later waits given
// fail = true return at once, so the kernel always runs to its end.  The fast
// path is one try_wait; the polling loop is out of line.
__device__ __noinline__ bool mbar_wait_slow(unsigned addr, unsigned parity, bool fail, int *err,
                                            unsigned long long limit_ns) {
    if (fail) return true;
    unsigned done = 0;
    unsigned long long t0 = 0;
    for (unsigned it = 0;; ++it) {
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(done) : "r"(addr), "r"(parity) : "memory");
        if (done) return false;
        if ((it & 63) == 0) {
            const unsigned long long now = global_ns();
            if (it == 0) t0 = now;
            else if (now - t0 > limit_ns) {
                if (err) atomicExch(err, 1);
                return true;
            }
        }
    }
}
__device__ __forceinline__ bool mbar_ready(unsigned addr, unsigned parity) {
    unsigned ready;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(ready) : "r"(addr), "r"(parity) : "memory");
    return ready != 0;
}
__device__ __forceinline__ void mbar_wait(unsigned addr, unsigned parity, bool &fail, int *err,
                                          unsigned long long limit_ns) {
    if (!mbar_ready(addr, parity)) fail = mbar_wait_slow(addr, parity, fail, err, limit_ns);
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// shared::cta -> shared::cluster bulk copy completing on the destination's mbarrier
__device__ __forceinline__ void bulk_copy_to_peer(unsigned dst, unsigned src, unsigned bytes, unsigned mbar) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "r"(src), "r"(bytes), "r"(mbar) : "memory");
}
__device__ __forceinline__ void st_async4(unsigned addr, float a, float b, float c, float d, unsigned mbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1,%2,%3,%4}, [%5];"
                 :: "r"(addr), "f"(a), "f"(b), "f"(c), "f"(d), "r"(mbar) : "memory");
}

// Per-thread view of one sequence's m buffers.
template <class C>
struct VitThread {
    static constexpr int K = C::K, NQ = C::NQ, NP = C::NP, NR = C::NR, R = C::R, CL = C::CL;
    u64 cwp[K][NP];          // codewords of the owned states s = k*Q + NQ*v + jq
    int v, slot;
    unsigned rank;
    unsigned rd0, wr0;       // byte offsets of this thread's first read / write

    // Layout of one (set, buffer).  CTA mode: m[f] of sequence `slot` at
    // chunk slot*Q/4 + f/4.  Cluster mode: each CTA holds the values its own
    // threads read -- m[k*Rn + r] lives in CTA r / (Rn/2) at local float
    // k*(Rn/2) + r % (Rn/2) -- so writers push (half of them remotely) and
    // every read is local.  Chunks are XOR-swizzled (bank-conflict free).
    __device__ __forceinline__ unsigned loc(int f) const {
        if (CL == 1) return unsigned(slot) * unsigned(C::Q) + unsigned(f);
        const int k = f / C::Rn, r = f % C::Rn;
        return unsigned(k * (C::Rn / 2) + (r % (C::Rn / 2)));
    }
    __device__ __forceinline__ unsigned off(int f) const {
        const unsigned l = loc(f);
        return (swz_chunk<R>(l >> 2) << 4) + ((l & 3u) << 2);
    }
    __device__ __forceinline__ int r0() const { return (NQ * v) >> R; }

    __device__ __forceinline__ void setup() {
        rd0 = off(r0());
        wr0 = off(NQ * v);
    }

    // m_{t-1} reads (always from this CTA's shared memory).
    __device__ __forceinline__ void load_prev(unsigned own, float (&m)[K][NR]) const {
        constexpr unsigned KS = unsigned(C::KSTRIDE * 4);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            if (NR >= 4) {
#pragma unroll
                for (int c4 = 0; c4 < NR / 4; ++c4) {
                    const unsigned o = C::FAST ? ((rd0 + unsigned(k) * KS) ^ (unsigned(c4) << 4))
                                               : off(k * C::Rn + r0() + 4 * c4);
                    const float4 q4 = lds4(own + o, false);
                    m[k][4 * c4 + 0] = q4.x; m[k][4 * c4 + 1] = q4.y;
                    m[k][4 * c4 + 2] = q4.z; m[k][4 * c4 + 3] = q4.w;
                }
            } else {
                const unsigned o = C::FAST ? (rd0 + unsigned(k) * KS) : off(k * C::Rn + r0());
                m[k][0] = lds1(own + o, false);
            }
        }
    }

    // One step for the owned q: writes m_t (at wbase + offset - wshift: the
    // local buffer, or the outbox for values the peer reads), returns the
    // thread's decision record (BPW words, low word first; the F-bit field
    // of q-local index jq in word jq / HQ at bits F (jq % HQ) .. + F).
    template <bool PREV>
    __device__ __forceinline__ u64 step(float x, const float (&m)[K][NR], unsigned wbase, unsigned wshift) const {
        constexpr int F = C::F, CPW = C::HQ / 4;    // decision bits per q, 4-q chunks per word
        const u64 xx = pk2(x, x);
        unsigned word[C::BPW];
        // chunks of 4 new m values (2 pairs) are stored as soon as they are
        // complete; each chunk packs its 4*F decision bits in its own word
        // (independent shift chains), merged with bit-field inserts
#pragma unroll
        for (int c4 = NQ / 4 - 1; c4 >= 0; --c4) {
            float mo[4];
            unsigned cw_bits = 0;
#pragma unroll
            for (int p = 2 * c4 + 1; p >= 2 * c4; --p) {
                const int i = (NQ >= K) ? ((2 * p) >> R) : 0;
                u64 c[K];
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    u64 d = sub2(xx, cwp[k][p]);
                    d = sq2(d);
                    c[k] = PREV ? add2(d, pk2(m[k][i], m[k][i])) : d;
                }
                if constexpr (C::RAW) {
                    // m = min over k (3-input mins), then s_k = sign(m - c_k):
                    // m - c_k is +0 exactly when c_k == m, negative otherwise
                    // (costs are never -0), so the lowest clear bit is the
                    // first-index argmin of trellis.py's torch.min; all-inf
                    // candidates give inf - inf = the canonical NaN (sign
                    // clear), i.e. k = 0 as torch picks
                    float lo[K], hi[K];
#pragma unroll
                    for (int k = 0; k < K; ++k) up2(c[k], lo[k], hi[k]);
                    float mlo, mhi;
                    if constexpr (K == 4) {
                        mlo = min3f(lo[0], lo[1], fminf(lo[2], lo[3]));
                        mhi = min3f(hi[0], hi[1], fminf(hi[2], hi[3]));
                    } else {
                        mlo = min3f(min3f(lo[0], lo[1], lo[2]), min3f(lo[3], lo[4], lo[5]), fminf(lo[6], lo[7]));
                        mhi = min3f(min3f(hi[0], hi[1], hi[2]), min3f(hi[3], hi[4], hi[5]), fminf(hi[6], hi[7]));
                    }
                    mo[2 * (p - 2 * c4)] = mlo;
                    mo[2 * (p - 2 * c4) + 1] = mhi;
                    // the pair's 2F bits interleave its two q: bit 2k holds s_k of
                    // the even q (low half), bit 2k + 1 that of the odd q, so
                    // each difference is packed as soon as it exists
                    const u64 mn = pk2(mlo, mhi);
#pragma unroll
                    for (int k = F - 1; k >= 0; --k) {
                        float el, eh;
                        up2(sub2(mn, c[k]), el, eh);
                        cw_bits = shift_in_sign(cw_bits, __float_as_uint(eh));
                        cw_bits = shift_in_sign(cw_bits, __float_as_uint(el));
                    }
                } else {
                    unsigned blo[R], bhi[R];
                    const u64 mn = tourney<R>(c, blo, bhi);
                    up2(mn, mo[2 * (p - 2 * c4)], mo[2 * (p - 2 * c4) + 1]);
#pragma unroll
                    for (int j = R - 1; j >= 0; --j) cw_bits = shift_in_sign(cw_bits, bhi[j]);
#pragma unroll
                    for (int j = R - 1; j >= 0; --j) cw_bits = shift_in_sign(cw_bits, blo[j]);
                }
            }
            const int w = c4 / CPW, sub = c4 % CPW;
            if (sub == CPW - 1) word[w] = cw_bits << (4 * F * sub);
            else word[w] = bfi(cw_bits, word[w], 4 * F * sub, 4 * F);
            const unsigned o = C::FAST ? (wr0 ^ (unsigned(c4) << 4)) : off(NQ * v + 4 * c4);
            sts4(wbase + o - wshift, mo[0], mo[1], mo[2], mo[3]);
        }
        if constexpr (C::BPW == 1) return u64(word[0]);
        else return u64(word[0]) | (u64(word[1]) << 32);
    }

    // Final step: costs of all owned states, first-index argmin.
    template <bool PREV>
    __device__ __forceinline__ void final_argmin(float x, const float (&m)[K][NR], float &bv, int &bi) const {
        const u64 xx = pk2(x, x);
        bi = NQ * v;  // valid even if every cost is NaN
#pragma unroll
        for (int k = 0; k < K; ++k) {
#pragma unroll
            for (int p = 0; p < NP; ++p) {
                const int i = (NQ >= K) ? ((2 * p) >> R) : 0;
                u64 d = sub2(xx, cwp[k][p]);
                d = sq2(d);
                if (PREV) d = add2(d, pk2(m[k][i], m[k][i]));
                float lo, hi;
                up2(d, lo, hi);
                const int s = k * C::Q + NQ * v + 2 * p;
                if (k == 0 && p == 0) bv = lo;
                else if (lo < bv) { bv = lo; bi = s; }
                if (hi < bv) { bv = hi; bi = s + 1; }
            }
        }
    }
};

__device__ __forceinline__ bool better(float v1, int i1, float v2, int i2) {
    return v1 < v2 || (v1 == v2 && i1 < i2);
}

// Synchronises the threads of one sequence (CTA mode).
template <class C>
__device__ __forceinline__ void seq_sync(int slot) {
    if (C::TPS <= 32) __syncwarp();
    else if (C::TPS == kThreads) __syncthreads();
    else asm volatile("bar.sync %0, %1;" :: "r"(1 + slot), "r"(C::TPS) : "memory");
}

// Timeouts of the cluster exchange (bounded mbarrier waits) are reported here.
__device__ int g_vit_timeout;
__device__ unsigned long long g_wait_limit_ns = 2000000000ull;

__device__ __noinline__ bool vit_wait_slow(unsigned addr, unsigned parity, bool fail) {
    return mbar_wait_slow(addr, parity, fail, &g_vit_timeout, g_wait_limit_ns);
}
// The Viterbi exchange's bounded wait (limit g_wait_limit_ns, flag g_vit_timeout).
__device__ __forceinline__ void vit_wait(unsigned addr, unsigned parity, bool &fail) {
    if (!mbar_ready(addr, parity)) fail = vit_wait_slow(addr, parity, fail);
}

template <class C>
__global__ void __cluster_dims__(C::CL, 1, 1) __launch_bounds__(kThreads, 1)
viterbi_fwd_kernel(VitArgs a) {
    constexpr int K = C::K, NQ = C::NQ, NR = C::NR, NSET = C::NSET, NP = C::NP, TPS = C::TPS, CL = C::CL;
    constexpr int NBUF = C::NBUF;
    extern __shared__ __align__(16) float sm_v[];
    __shared__ float red_v[NSET][kThreads / 32];
    __shared__ int red_i[NSET][kThreads / 32];
    __shared__ __align__(8) unsigned long long full[NSET][NBUF];   // cluster mode: step's inputs complete
    __shared__ unsigned done_cnt[NSET][NBUF];                       // cluster mode: warps done with a step

    VitThread<C> th;
    const int tid = threadIdx.x;
    int64_t seq_base;
    if (CL == 1) {
        th.rank = 0;
        th.slot = tid / TPS;
        th.v = tid % TPS;
        seq_base = int64_t(blockIdx.x) * C::SPS;
    } else {
        th.rank = cluster_rank();
        th.slot = 0;
        th.v = int(th.rank) * kThreads + tid;
        seq_base = int64_t(blockIdx.x / CL) * NSET;
    }
    th.setup();
#pragma unroll
    for (int k = 0; k < K; ++k)
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            const int s = k * C::Q + NQ * th.v + 2 * p;
            th.cwp[k][p] = pk2(__ldg(a.cw + s), __ldg(a.cw + s + 1));
        }

    const unsigned smem0 = unsigned(__cvta_generic_to_shared(sm_v));
    constexpr unsigned BUF = unsigned(C::FLOATS * 4);
    // cluster mode: outboxes follow the buffers; the peer's share of this
    // thread's outputs (bit TBIT of v names the reading CTA) goes there
    const unsigned obox0 = smem0 + unsigned(NSET * NBUF) * BUF;   // (cluster mode; derived where used)
    const bool wremote = CL == 2 && (((th.v >> C::TBIT) & 1) != int(th.rank));
    const unsigned half_off = th.rank * C::OBYTES;     // this CTA produces half `rank` of each buffer
    const unsigned full0 = unsigned(__cvta_generic_to_shared(&full[0][0]));
    // where this thread's step outputs go: the local buffer, or (values the
    // peer reads) the outbox, whose offset 0 is the peer's half `rank`
    const unsigned wbase0 = wremote ? obox0 - half_off : smem0;
    const unsigned wstep = wremote ? unsigned(C::OBYTES) : BUF;
    bool fail = false;

    // set X is sequence first + X (cluster mode) or first (CTA mode, one set);
    // the sets' inputs and backpointers are at fixed offsets from set 0's, so
    // one input pointer, one backpointer pointer and a validity mask carry
    // them (registers are at the 128 limit)
    const int64_t first = seq_base + (CL == 1 ? th.slot : 0);
    // 32-bit sequence strides (T * TPS < 2^32) except in the L = 16, R = 3
    // form, whose register allocation is better with 64-bit ones (measured:
    // L = 16 R = 2 55.2 -> 56.2 % of the lane peak, R = 3 54.1 -> 53.2 %)
    using Off = typename std::conditional<C::CL == 2 && C::R == 3, int64_t, unsigned>::type;
    const Off bstride = Off(a.T - 1) * Off(TPS);
    unsigned vmask = 0;
#pragma unroll
    for (int X = 0; X < NSET; ++X) vmask |= (first + X < a.nbatch ? 1u : 0u) << X;
    const float *xcur = a.xn + (a.seq0 + (vmask & 1u ? first : 0)) * int64_t(a.T);
    // one record (BPW words, low word first) per thread and step
    using Rec = typename std::conditional<C::BPW == 2, u64, uint32_t>::type;
    Rec *bcur = reinterpret_cast<Rec *>(a.bp) + (vmask & 1u ? first : 0) * int64_t(bstride) + th.v;
    float xv[NSET];
#pragma unroll
    for (int X = 0; X < NSET; ++X) xv[X] = (vmask >> X) & 1u ? __ldg(xcur + Off(X) * Off(a.T)) : 0.f;

    if (CL == 2) {
        if (tid < NSET * NBUF) {
            // phase completes on: the arm (arrive + expect_tx; here for phase 0,
            // later by the last warp of the step that read the buffer), the last
            // local warp's arrival (all local writes of the step done) and the
            // peer's bulk copy (OBYTES of transaction)
            mbar_init(full0 + unsigned(tid) * 8u, 2);
            mbar_expect_tx(full0 + unsigned(tid) * 8u, C::OBYTES);   // arm phase 0
            done_cnt[tid / NBUF][tid % NBUF] = 0u;
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        cluster_arrive();      // peers running and barriers initialised before any copy
        cluster_wait();
    }

    float m[K][NR];
#pragma unroll (C::UNROLL)
    for (int t = 0; t + 1 < a.T; ++t) {
#pragma unroll
        for (int X = 0; X < NSET; ++X) {
            const float x = xv[X];
            // (the L = 16 R = 3 form measured 54.4 % with this association
            // of the offset, 53.9 % with the one below)
            if constexpr (sizeof(Off) == 8)
                xv[X] = (vmask >> X) & 1u ? __ldg(xcur + X * int64_t(a.T) + t + 1) : 0.f;
            else
                xv[X] = (vmask >> X) & 1u ? __ldg(xcur + (Off(X) * Off(a.T) + Off(t + 1))) : 0.f;
            Rec word;
            if (CL == 1) {
                const unsigned wb = smem0 + unsigned(X * NBUF + (t & 1)) * BUF;
                if (t == 0) {
                    word = Rec(th.template step<false>(x, m, wb, 0u));
                } else {
                    th.load_prev(smem0 + unsigned(X * NBUF + ((t - 1) & 1)) * BUF, m);
                    word = Rec(th.template step<true>(x, m, wb, 0u));
                }
                seq_sync<C>(th.slot);
            } else {
                const int jw = t & 1;
                // local values into buffer jw, the peer's share into outbox jw
                const unsigned wb = wbase0 + unsigned(X * NBUF + jw) * wstep;
                const unsigned wsh = 0u;
                if (t == 0) {
                    word = Rec(th.template step<false>(x, m, wb, wsh));
                } else {
                    const int jr = (t - 1) & 1;
                    const unsigned mbr = full0 + unsigned(X * NBUF + jr) * 8u;
                    vit_wait(mbr, unsigned(((t - 1) >> 1) & 1), fail);
                    th.load_prev(smem0 + unsigned(X * NBUF + jr) * BUF, m);
                    word = Rec(th.template step<true>(x, m, wb, wsh));
                }
                if (wremote) fence_proxy_async_smem();   // outbox writes -> async proxy
                // no CTA barrier: the last warp to finish the step ships the
                // outbox and releases the local half; warps can run up to one
                // step apart (a warp at step t+1 has waited for every warp's
                // step t, which orders all reuse of buffers and outboxes)
                __syncwarp();
                if ((tid & 31) == 0) {
                    // acq_rel: releases this warp's step, acquires all earlier warps'
                    unsigned old;
                    asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                                 : "=r"(old) : "r"(unsigned(__cvta_generic_to_shared(&done_cnt[X][jw]))) : "memory");
                    if ((old % (kThreads / 32)) == kThreads / 32 - 1) {
                        // every warp has passed its wait on the buffer read in
                        // this step: arm that buffer's next phase (before the
                        // copy below, which the peer's next copy into it follows)
                        if (t > 0) mbar_expect_tx(full0 + unsigned(X * NBUF + ((t - 1) & 1)) * 8u, C::OBYTES);
                        bulk_copy_to_peer(mapa_shared(smem0 + unsigned(X * NBUF + jw) * BUF + half_off, th.rank ^ 1u),
                                          obox0 + unsigned(X * NBUF + jw) * C::OBYTES, C::OBYTES,
                                          mapa_shared(full0 + unsigned(X * NBUF + jw) * 8u, th.rank ^ 1u));
                        mbar_arrive(full0 + unsigned(X * NBUF + jw) * 8u);
                    }
                }
            }
            if ((vmask >> X) & 1u) bcur[Off(X) * bstride] = word;
        }
        bcur += TPS;
    }
    // final step: argmin over all states of cost_{T-1}
#pragma unroll
    for (int X = 0; X < NSET; ++X) {
        float bv;
        int bi;
        if (a.T == 1) {
            th.template final_argmin<false>(xv[X], m, bv, bi);
        } else {
            const int jr = (a.T - 2) & 1;
            if (CL == 2)
                vit_wait(full0 + unsigned(X * NBUF + jr) * 8u, unsigned(((a.T - 2) >> 1) & 1), fail);
            th.load_prev(smem0 + unsigned(X * NBUF + jr) * BUF, m);
            th.template final_argmin<true>(xv[X], m, bv, bi);
        }
        constexpr int segw = TPS < 32 ? TPS : 32;
#pragma unroll
        for (int o = 1; o < segw; o <<= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (TPS <= 32) {
            if ((tid % TPS) == 0 && ((vmask >> X) & 1u)) a.fin[first + X] = bi;
        } else if ((tid & 31) == 0) {
            red_v[X][tid >> 5] = bv;
            red_i[X][tid >> 5] = bi;
        }
    }
    if (TPS > 32) {
        if (CL == 1) {
            __syncthreads();
            if ((tid % TPS) == 0) {
                constexpr int wps = TPS / 32;
                const int w0 = tid >> 5;
                float bv = red_v[0][w0];
                int bi = red_i[0][w0];
                for (int w = 1; w < wps; ++w)
                    if (better(red_v[0][w0 + w], red_i[0][w0 + w], bv, bi)) { bv = red_v[0][w0 + w]; bi = red_i[0][w0 + w]; }
                if (vmask & 1u) a.fin[first] = bi;
            }
        } else {
            cluster_arrive();
            cluster_wait();
            if (th.rank == 0 && tid == 0) {
#pragma unroll
                for (int X = 0; X < NSET; ++X) {
                    float bv = red_v[X][0];
                    int bi = red_i[X][0];
                    for (int w = 1; w < kThreads / 32; ++w)
                        if (better(red_v[X][w], red_i[X][w], bv, bi)) { bv = red_v[X][w]; bi = red_i[X][w]; }
                    const unsigned rv = mapa_shared(unsigned(__cvta_generic_to_shared(&red_v[X][0])), 1u);
                    const unsigned ri = mapa_shared(unsigned(__cvta_generic_to_shared(&red_i[X][0])), 1u);
                    for (int w = 0; w < kThreads / 32; ++w) {
                        float ov;
                        int oi;
                        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(ov) : "r"(rv + 4u * w));
                        asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(oi) : "r"(ri + 4u * w));
                        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                    }
                    if ((vmask >> X) & 1u) a.fin[first + X] = bi;
                }
            }
            cluster_arrive();   // keep shared memory alive for the peer's reads
            cluster_wait();
        }
    }
}

// ---- packed codes --------------------------------------------------------------
// A state path is a shift register, s_t = ((s_{t-1} << R) | b_t) mod 2^L, so the
// bit string S = s_0 2^(R(T-1)) + sum_{t>=1} b_t 2^(R(T-1-t)), b_t = s_t mod 2^R,
// holds it in L + R (T-1) bits, and s_t = (S >> R(T-1-t)) mod 2^L.  S is stored
// least significant word first, words_per_seq 32-bit words per sequence.
__global__ void pack_kernel(const int32_t *states, int64_t nseq, int T, int L, int R, int words,
                            uint32_t *packed) {
    const int64_t total = nseq * words;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t sq = i / words;
        const int w = int(i % words);
        const int32_t *st = states + sq * T;
        const int lo = 32 * w, hi = lo + 32;      // bit range of this word
        uint64_t acc = 0;
        // s_0 at offset R (T-1), width L
        {
            const int off = R * (T - 1);
            if (off < hi && off + L > lo) {
                const uint64_t v = uint64_t(uint32_t(st[0]) & ((1u << L) - 1u));
                acc |= off >= lo ? (v << (off - lo)) : (v >> (lo - off));
            }
        }
        // b_t at offset R (T-1-t), width R: t with the field overlapping [lo, hi)
        const int t_first = max(1, T - 1 - (hi - 1) / R);
        const int t_last = min(T - 1, T - 1 - (lo - R + 1 > 0 ? (lo - R + 1 + R - 1) / R : 0));
        for (int t = t_first; t <= t_last; ++t) {
            const int off = R * (T - 1 - t);
            if (off >= hi || off + R <= lo) continue;
            const uint64_t v = uint64_t(uint32_t(st[t]) & ((1u << R) - 1u));
            acc |= off >= lo ? (v << (off - lo)) : (v >> (lo - off));
        }
        packed[i] = uint32_t(acc);
    }
}

__global__ void unpack_kernel(const uint32_t *packed, int64_t nseq, int T, int L, int R, int words, int32_t *states) {
    const int64_t total = nseq * T;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t sq = i / T;
        const int t = int(i % T);
        const int off = R * (T - 1 - t);
        const uint32_t *p = packed + sq * words;
        const int w = off >> 5;
        uint64_t v = __ldg(p + w);
        if (w + 1 < words) v |= uint64_t(__ldg(p + w + 1)) << 32;
        states[i] = int32_t((v >> (off & 31)) & ((1ull << L) - 1ull));
    }
}

// Self-test of the bounded wait: waits on an mbarrier phase that nothing
// completes; the wait gives up after limit_ns and reports it in *status.
__global__ void wait_timeout_probe_kernel(unsigned long long limit_ns, int *status) {
    __shared__ __align__(8) unsigned long long bar;
    const unsigned addr = unsigned(__cvta_generic_to_shared(&bar));
    if (threadIdx.x == 0) mbar_init(addr, 1);
    __syncthreads();
    bool fail = false;
    mbar_wait(addr, 0u, fail, status, limit_ns);
    __syncthreads();
    if (threadIdx.x == 0) mbar_arrive(addr);   // complete the phase before exit
}

// Traceback: one thread per sequence walks the decision records (the
// record layout of VitCfg: F-bit field of q-local jq in word jq / HQ).
template <int R>
__global__ void traceback_kernel(const uint32_t *bp, const int32_t *fin, int64_t nbatch, int T, int L,
                                 int32_t *states, int64_t seq0) {
    using C = VitCfg<(2 * R > 6 ? 2 * R : 6), R, 1>;     // record constants depend on R only
    constexpr int K = 1 << R, NQ = C::NQ, F = C::F, BPW = C::BPW, HQ = C::HQ;
    const int64_t sq = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
    if (sq >= nbatch) return;
    const int Q = 1 << (L - R);
    const int TPS = Q / NQ;
    const uint32_t *b = bp + sq * int64_t(T - 1) * TPS * BPW;
    int32_t *out = states + (seq0 + sq) * int64_t(T);
    int s = fin[sq] & ((1 << L) - 1);
    out[T - 1] = s;
    for (int t = T - 1; t >= 1; --t) {
        const int q = s >> R;
        const int jq = q % NQ;
        const uint32_t w = __ldg(b + (int64_t(t - 1) * TPS + q / NQ) * BPW + jq / HQ);
        int k;
        if constexpr (C::RAW) {
            // s_k at bit 2k of the shifted pair bits; the lowest clear one is
            // the first minimum (K - 1 if none)
            const unsigned bits = w >> (2 * F * ((jq % HQ) >> 1) + (jq & 1));
            k = F;
#pragma unroll
            for (int j = F - 1; j >= 0; --j)
                if (!((bits >> (2 * j)) & 1u)) k = j;
        } else {
            k = int((w >> (F * (jq % HQ))) & ((1u << F) - 1u));
        }
        s = k * Q + q;
        out[t - 1] = s;
    }
}

template <int L, int R>
int launch_viterbi(const VitArgs &a, cudaStream_t st) {
    constexpr int CL = L == 16 ? 2 : 1;
    using C = VitCfg<L, R, CL>;
    const size_t smem = size_t(C::NSET) * C::NBUF * (C::FLOATS + C::OFLOATS) * sizeof(float);
    auto kern = viterbi_fwd_kernel<C>;
    if (uq::set_smem_attr(reinterpret_cast<const void *>(kern), int(smem)) != cudaSuccess)
        return uq::check_cuda("viterbi: set smem attribute");
    int64_t ctas;
    if (CL == 1) ctas = (a.nbatch + C::SPS - 1) / C::SPS;
    else ctas = (a.nbatch + C::NSET - 1) / C::NSET * CL;
    if (ctas > 0) { uq::ProfScope _p("viterbi_fwd", st); kern<<<unsigned(ctas), kThreads, smem, st>>>(a); }
    return uq::check_cuda("viterbi_fwd_kernel launch");
}

// Sequences that one wave of resident CTAs (clusters for L = 16) covers, or 0
// if the occupancy query fails.  Batches that are whole multiples of it leave
// no partly filled last wave (2,048-sequence batches at L = 16 ran 13.84
// waves of 74 clusters: 1.1 % of the cluster slots idle).
template <int L, int R>
int64_t viterbi_wave() {
    constexpr int CL = L == 16 ? 2 : 1;
    using C = VitCfg<L, R, CL>;
    const size_t smem = size_t(C::NSET) * C::NBUF * (C::FLOATS + C::OFLOATS) * sizeof(float);
    auto kern = viterbi_fwd_kernel<C>;
    if (uq::set_smem_attr(reinterpret_cast<const void *>(kern), int(smem)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (CL == 1) {
        int per_sm = 0;
        if (uq::occupancy_blocks(&per_sm, reinterpret_cast<const void *>(kern), kThreads, smem) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        return int64_t(per_sm) * uq::num_sms() * C::SPS;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(CL * 64), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    int ncl = 0;
    if (uq::occupancy_clusters(&ncl, reinterpret_cast<const void *>(kern), &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return int64_t(ncl) * C::NSET;
}

template <int R, int L>
int64_t wave_l(int Lrt) {
    if constexpr (L > 16) {
        return 0;
    } else {
        if (Lrt == L) return viterbi_wave<L, R>();
        return wave_l<R, L + 1>(Lrt);
    }
}

template <int R, int L>
int dispatch_l(int Lrt, const VitArgs &a, cudaStream_t st) {
    if constexpr (L > 16) {
        return uq::fail(UQ_ERR_UNSUPPORTED, "viterbi: L=%d", Lrt);
    } else {
        if (Lrt == L) return launch_viterbi<L, R>(a, st);
        return dispatch_l<R, L + 1>(Lrt, a, st);
    }
}

template <int R>
int run_viterbi_r(const float *xn, int64_t nseq, int T, int L, const float *cw, int32_t *states,
                  uint32_t *bp, int32_t *fin, int64_t batch, cudaStream_t st) {
    constexpr int LMIN = (2 * R > 6) ? 2 * R : 6;
    if (batch < nseq) {
        const int64_t wave = wave_l<R, LMIN>(L);
        if (wave > 0 && batch > wave) batch = batch / wave * wave;
    }
    for (int64_t s0 = 0; s0 < nseq; s0 += batch) {
        VitArgs a{};
        a.xn = xn; a.seq0 = s0; a.nbatch = std::min<int64_t>(batch, nseq - s0);
        a.T = T; a.cw = cw; a.bp = bp; a.fin = fin;
        int rc = dispatch_l<R, LMIN>(L, a, st);
        if (rc) return rc;
        const int64_t g = (a.nbatch + 127) / 128;
        { uq::ProfScope _p("traceback", st); traceback_kernel<R><<<unsigned(g), 128, 0, st>>>(bp, fin, a.nbatch, T, L, states, s0); }
        if ((rc = uq::check_cuda("traceback_kernel launch"))) return rc;
    }
    return UQ_OK;
}

__global__ void decode_kernel(const int32_t *states, const float *cw, const float *sc, int64_t group,
                              int64_t ntot, float *out) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < ntot; i += int64_t(gridDim.x) * blockDim.x)
        out[i] = __fmul_rn(__ldg(cw + __ldg(states + i)), __ldg(sc + i / group));
}

__global__ void decode_rows_kernel(const int32_t *states, const float *cw, const float *sc, int64_t nrow,
                                   int64_t T, int64_t Tp, int64_t group, float *out) {
    const int64_t n = nrow * T;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / T, c = i - r * T;
        const int64_t j = r * Tp + c;
        out[i] = __fmul_rn(__ldg(cw + __ldg(states + j)), __ldg(sc + j / group));
    }
}

int vit_check(int64_t nseq, int T, int L, int R) {
    if (nseq < 0 || T < 1) return uq::fail(UQ_ERR_INVALID, "viterbi: bad nseq / T");
    if (R < 1 || R > 4 || L > 16 || L < 6 || L < 2 * R)
        return uq::fail(UQ_ERR_UNSUPPORTED, "viterbi: (L=%d, R=%d) not built (need 1<=R<=4, max(6,2R)<=L<=16)", L, R);
    return UQ_OK;
}

}  // namespace

namespace uq {

int vit_record_words(int R) {
    switch (R) {
        case 1: return VitCfg<6, 1, 1>::BPW;
        case 2: return VitCfg<6, 2, 1>::BPW;
        case 3: return VitCfg<6, 3, 1>::BPW;
        case 4: return VitCfg<8, 4, 1>::BPW;
    }
    return 1;
}

int64_t vit_seq_bytes(int T, int L, int R) {
    // decision records per sequence: (T-1) * 2^L / 64 of vit_record_words(R)
    // 32-bit words, plus the final state
    return int64_t(T - 1) * ((int64_t(1) << L) / 64) * 4 * vit_record_words(R) + 4;
}

size_t trellis_ws_bytes(int64_t nseq, int T, int L, int R) {
    // cap the backpointer batch at ~8 GiB per record word (whole sequences,
    // at least one launch worth of sequences): each batch ends with a
    // traceback launch that is latency bound (~0.19 ms whatever its size),
    // so larger batches mean fewer of them (at L = 16, T = 256: ~8,200
    // sequences per batch)
    const int64_t per = vit_seq_bytes(T, L, R);
    int64_t want = nseq;
    const int64_t cap = (int64_t(8) << 30) * vit_record_words(R) / per;
    const int64_t min_batch = 2 * 148;
    if (want > cap) want = std::max<int64_t>(cap, min_batch);
    return size_t(std::max<int64_t>(want, 1) * per) + 512;
}

int trellis_viterbi(const float *xn, int64_t nseq, int T, int L, int R, const float *cw, int32_t *states,
                    void *ws, size_t ws_bytes, cudaStream_t st) {
    NvtxRange _r("trellis_viterbi");
    const int64_t per = vit_seq_bytes(T, L, R);
    int64_t batch = int64_t((ws_bytes > 512 ? ws_bytes - 512 : 0) / size_t(per));
    if (batch < 1) return fail(UQ_ERR_WORKSPACE, "viterbi: workspace %zu too small (need %lld per sequence)",
                               ws_bytes, (long long)per);
    if (batch > nseq) batch = nseq;
    Carver c(ws, ws_bytes);
    int32_t *fin = c.take<int32_t>(size_t(batch));
    uint32_t *bp = c.take<uint32_t>(size_t(batch) * size_t(T - 1) * ((size_t(1) << L) / 64) * vit_record_words(R));
    switch (R) {
        case 1: return run_viterbi_r<1>(xn, nseq, T, L, cw, states, bp, fin, batch, st);
        case 2: return run_viterbi_r<2>(xn, nseq, T, L, cw, states, bp, fin, batch, st);
        case 3: return run_viterbi_r<3>(xn, nseq, T, L, cw, states, bp, fin, batch, st);
        case 4: return run_viterbi_r<4>(xn, nseq, T, L, cw, states, bp, fin, batch, st);
    }
    return fail(UQ_ERR_UNSUPPORTED, "viterbi: R");
}

int trellis_normalize(const void *A, int dtype, int64_t nrow, int64_t T, int64_t lda, int64_t Tp, int64_t group,
                      float *xn, float *sc, cudaStream_t st) {
    NvtxRange _r("trellis_normalize");
    NormArgs a{};
    a.A = A; a.dtype = dtype; a.nrow = nrow; a.T = T; a.lda = lda; a.Tp = Tp; a.group = int(group);
    a.xn = xn; a.sc = sc;
    return launch_normalize(a, st);
}

int trellis_decode(const int32_t *states, const float *cw, const float *sc, int64_t group, int64_t ntot,
                   float *out, cudaStream_t st) {
    NvtxRange _r("trellis_decode");
    const int grid = int(std::max<int64_t>(1, std::min<int64_t>((ntot + 255) / 256, int64_t(num_sms()) * 16)));
    if (ntot > 0) { uq::ProfScope _p("decode", st); decode_kernel<<<grid, 256, 0, st>>>(states, cw, sc, group, ntot, out); }
    return check_cuda("decode_kernel launch");
}

}  // namespace uq

// ---------------------------------------------------------------------------
// Scratch-free Viterbi entry point.
//
// Some callers cannot allocate device memory: a host program that hands its
// whole GPU memory to its own allocator and exposes no allocation hook to
// plug-ins, or a latency-sensitive caller that must never hit cudaMalloc's
// device-wide synchronisation.  For them uq_trellis_viterbi_noalloc keeps the
// backpointer scratch in a fixed file-scope device array instead of a caller
// workspace.  The array is created when the library's module is loaded on a
// device and is held by every GPU that loads the library until the process
// exits.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;   // 64 MiB per device
// Cached device addresses of the scratch array, one per (device, context).
// The array lives in the library's module, which the runtime loads into every
// context that uses it, so a new context on the same device (after
// cudaDeviceReset, or a caller's own context) has its own copy.  Contexts are
// told apart by the driver's context ID, which is unique for the life of the
// process (a context handle may be reused after its context is destroyed).
struct NoAllocSlot {
    int dev = -1;
    unsigned long long ctx_id = 0;
    void *ptr = nullptr;
};
constexpr int kNoAllocSlots = 64;
std::mutex g_noalloc_mu;
NoAllocSlot g_noalloc_slot[kNoAllocSlots];
int g_noalloc_next = 0;

// cuCtxGetCurrent / cuCtxGetId from the driver, fetched through the runtime
// (the library links only the CUDA runtime); null if the driver lacks them.
typedef int (*CtxGetCurrentFn)(void **);
typedef int (*CtxGetIdFn)(void *, unsigned long long *);
struct CtxQuery {
    CtxGetCurrentFn current = nullptr;
    CtxGetIdFn id = nullptr;
};
const CtxQuery &ctx_query() {
    static std::once_flag once;
    static CtxQuery q;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult r = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &r) == cudaSuccess &&
            r == cudaDriverEntryPointSuccess)
            q.current = reinterpret_cast<CtxGetCurrentFn>(p);
        p = nullptr;
        r = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &r) == cudaSuccess &&
            r == cudaDriverEntryPointSuccess)
            q.id = reinterpret_cast<CtxGetIdFn>(p);
        cudaGetLastError();
    });
    return q;
}

// ID of the context current on this thread, 0 if none is bound or the
// driver cannot say.
unsigned long long current_ctx_id() {
    const CtxQuery &q = ctx_query();
    void *ctx = nullptr;
    unsigned long long id = 0;
    if (!q.current || !q.id || q.current(&ctx) != 0 || !ctx || q.id(ctx, &id) != 0) return 0;
    return id;
}
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array in the current context, looked up with
// cudaGetSymbolAddress on the first call per (device, context) and cached
// (host code may not use the symbol itself as a device address).
static int noalloc_scratch(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return uq::check_cuda("noalloc: cudaGetDevice");
    unsigned long long id = current_ctx_id();
    if (id) {
        std::lock_guard<std::mutex> g(g_noalloc_mu);
        for (const NoAllocSlot &s : g_noalloc_slot)
            if (s.ptr && s.dev == dev && s.ctx_id == id) {
                *out = s.ptr;
                return UQ_OK;
            }
    }
    // first call in this context (or no context bound to the thread yet: the
    // lookup binds the runtime's context, whose ID is then cached)
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
        return uq::fail(UQ_ERR_CUDA, "noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    id = current_ctx_id();
    if (id) {   // without a context ID nothing is cached: every call looks the address up
        std::lock_guard<std::mutex> g(g_noalloc_mu);
        g_noalloc_slot[g_noalloc_next++ % kNoAllocSlots] = NoAllocSlot{dev, id, p};
    }
    *out = p;
    return UQ_OK;
}

extern "C" {

size_t uq_trellis_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int uq_trellis_viterbi_noalloc(const float *xn, int64_t nseq, int T, int L, int R, const float *cw,
                               int32_t *states, void *stream) {
    int rc = vit_check(nseq, T, L, R);
    if (rc) return rc;
    const int64_t per = uq::vit_seq_bytes(T, L, R);
    if (size_t(per) + 512 > kNoAllocScratchBytes)
        return uq::fail(UQ_ERR_INVALID,
                        "uq_trellis_viterbi_noalloc: one sequence (T=%d, L=%d) needs %lld bytes of backpointer "
                        "scratch, more than the %zu-byte static array; use uq_trellis_viterbi with a workspace",
                        T, L, (long long)per, kNoAllocScratchBytes);
    if (nseq == 0) return UQ_OK;
    if (!xn || !cw || !states) return uq::fail(UQ_ERR_INVALID, "uq_trellis_viterbi_noalloc: null pointer");
    void *scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch))) return rc;
    // The backpointers and final states are fully written before they are
    // read, so nothing in the array needs clearing between calls.
    return uq::trellis_viterbi(xn, nseq, T, L, R, cw, states, scratch, kNoAllocScratchBytes, UQ_STREAM(stream));
}

int uq_device_errors(void *stream) {
    if (cudaStreamSynchronize(UQ_STREAM(stream)) != cudaSuccess) return uq::check_cuda("uq_device_errors");
    int flag = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&flag, g_vit_timeout, sizeof(int)) != cudaSuccess) return uq::check_cuda("read timeout flag");
    if (flag) {
        cudaMemcpyToSymbol(g_vit_timeout, &zero, sizeof(int));
        return uq::fail(UQ_ERR_TIMEOUT, "a bounded device wait of the Viterbi cluster exchange timed out");
    }
    const int rto = uq::rht_take_timeout(), eto = uq::e8_take_timeout();
    if (rto < 0 || eto < 0) return uq::check_cuda("read tensor-map timeout flags");
    if (rto || eto) return uq::fail(UQ_ERR_TIMEOUT, "a bounded device wait of a tensor-map kernel timed out");
    const int bad = uq::qat_take_bad_state();
    if (bad < 0) return uq::check_cuda("read decoder state flag");
    if (bad) return uq::fail(UQ_ERR_INVALID, "a trellis state given to the decoder lies outside the codebook");
    return UQ_OK;
}

int uq_inject_device_flag(int which) {
    int rc = -1;
    if (which == 0) {
        const int one = 1;
        rc = cudaMemcpyToSymbol(g_vit_timeout, &one, sizeof(int)) == cudaSuccess ? 0 : -1;
    } else if (which == 1) {
        rc = uq::rht_set_timeout();
    } else if (which == 2) {
        rc = uq::e8_set_timeout();
    } else {
        return uq::fail(UQ_ERR_INVALID, "uq_inject_device_flag: which=%d not in {0, 1, 2}", which);
    }
    return rc ? uq::check_cuda("uq_inject_device_flag") : UQ_OK;
}

int uq_wait_timeout_selftest(double limit_ms, void *stream) {
    if (!(limit_ms > 0.0) || limit_ms > 2000.0) return uq::fail(UQ_ERR_INVALID, "limit_ms must be in (0, 2000]");
    cudaStream_t st = UQ_STREAM(stream);
    int *d = nullptr;
    if (cudaMallocAsync(&d, sizeof(int), st) != cudaSuccess) return uq::check_cuda("selftest alloc");
    cudaMemsetAsync(d, 0, sizeof(int), st);
    { uq::ProfScope _p("wait_probe", st); wait_timeout_probe_kernel<<<1, 32, 0, st>>>((unsigned long long)(limit_ms * 1e6), d); }
    int rc = uq::check_cuda("wait_timeout_probe_kernel launch");
    int flag = 0;
    cudaMemcpyAsync(&flag, d, sizeof(int), cudaMemcpyDeviceToHost, st);
    cudaFreeAsync(d, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) return uq::check_cuda("selftest sync");
    if (rc) return rc;
    return flag ? uq::fail(UQ_ERR_TIMEOUT, "bounded wait gave up as intended") : UQ_OK;
}

int uq_trellis_codebook(int L, float *out, void *stream) {
    if (L < 1 || L > 16) return uq::fail(UQ_ERR_UNSUPPORTED, "uq_trellis_codebook: L=%d not in [1, 16]", L);
    if (!out) return uq::fail(UQ_ERR_INVALID, "uq_trellis_codebook: null pointer");
    const int S = 1 << L;
    { uq::ProfScope _p("codebook", UQ_STREAM(stream)); codebook_kernel<<<(S + 255) / 256, 256, 0, UQ_STREAM(stream)>>>(L, out); }
    return uq::check_cuda("codebook_kernel launch");
}

int uq_trellis_normalize(const void *A, int a_dtype, int64_t ntot, int64_t group, int64_t seg, float *xn,
                         float *sc, void *stream) {
    if (ntot < 0 || group < 8 || group % 8 || group > 8192 || seg < 1 || !uq::dtype_size(a_dtype))
        return uq::fail(group % 8 || group > 8192 ? UQ_ERR_UNSUPPORTED : UQ_ERR_INVALID,
                        "uq_trellis_normalize: bad arguments (ntot=%lld group=%lld seg=%lld)",
                        (long long)ntot, (long long)group, (long long)seg);
    const int64_t padded = (ntot + group - 1) / group * group;
    if (padded % seg) return uq::fail(UQ_ERR_INVALID, "uq_trellis_normalize: padded size %lld not divisible by seg %lld",
                                      (long long)padded, (long long)seg);
    if (padded == 0) return UQ_OK;
    if (!A || !xn || !sc) return uq::fail(UQ_ERR_INVALID, "uq_trellis_normalize: null pointer");
    return uq::trellis_normalize(A, a_dtype, 1, ntot, ntot, padded, group, xn, sc, UQ_STREAM(stream));
}

int uq_trellis_normalize_rows(const void *A, int a_dtype, int64_t nrow, int64_t T, int64_t lda, int64_t group,
                              float *xn, float *sc, void *stream) {
    if (nrow < 0 || T < 1 || lda < T || group < 8 || group % 8 || group > 8192 || !uq::dtype_size(a_dtype))
        return uq::fail(UQ_ERR_INVALID, "uq_trellis_normalize_rows: bad arguments");
    if (nrow == 0) return UQ_OK;
    if (!A || !xn || !sc) return uq::fail(UQ_ERR_INVALID, "uq_trellis_normalize_rows: null pointer");
    const int64_t Tp = (T + group - 1) / group * group;
    return uq::trellis_normalize(A, a_dtype, nrow, T, lda, Tp, group, xn, sc, UQ_STREAM(stream));
}

size_t uq_trellis_workspace_bytes(int64_t nseq, int T, int L, int R) {
    if (vit_check(nseq, T, L, R) != UQ_OK) return 0;
    return uq::trellis_ws_bytes(nseq, T, L, R);
}

int uq_trellis_viterbi(const float *xn, int64_t nseq, int T, int L, int R, const float *cw, int32_t *states,
                       void *workspace, size_t workspace_bytes, void *stream) {
    int rc = vit_check(nseq, T, L, R);
    if (rc) return rc;
    if (nseq == 0) return UQ_OK;
    if (!xn || !cw || !states || !workspace) return uq::fail(UQ_ERR_INVALID, "uq_trellis_viterbi: null pointer");
    return uq::trellis_viterbi(xn, nseq, T, L, R, cw, states, workspace, workspace_bytes, UQ_STREAM(stream));
}

int uq_trellis_decode(const int32_t *states, const float *cw, const float *sc, int64_t group, int64_t ntot,
                      float *out, void *stream) {
    if (ntot < 0 || group < 1) return uq::fail(UQ_ERR_INVALID, "uq_trellis_decode: bad arguments");
    if (ntot == 0) return UQ_OK;
    if (!states || !cw || !sc || !out) return uq::fail(UQ_ERR_INVALID, "uq_trellis_decode: null pointer");
    return uq::trellis_decode(states, cw, sc, group, ntot, out, UQ_STREAM(stream));
}

int uq_trellis_decode_rows(const int32_t *states, const float *cw, const float *sc, int64_t nrow, int64_t T,
                           int64_t Tp, int64_t group, float *out, void *stream) {
    if (nrow < 0 || T < 1 || Tp < T || group < 1 || Tp % group)
        return uq::fail(UQ_ERR_INVALID, "uq_trellis_decode_rows: bad arguments");
    if (nrow == 0) return UQ_OK;
    if (!states || !cw || !sc || !out) return uq::fail(UQ_ERR_INVALID, "uq_trellis_decode_rows: null pointer");
    const int64_t n = nrow * T;
    const int grid = int(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, int64_t(uq::num_sms()) * 16)));
    { uq::ProfScope _p("decode_rows", UQ_STREAM(stream)); decode_rows_kernel<<<grid, 256, 0, UQ_STREAM(stream)>>>(states, cw, sc, nrow, T, Tp, group, out); }
    return uq::check_cuda("decode_rows_kernel launch");
}

int64_t uq_trellis_packed_words(int T, int L, int R) {
    if (T < 1 || L < 1 || L > 16 || R < 1 || R > 4 || R > L) return 0;
    return (int64_t(L) + int64_t(R) * (T - 1) + 31) / 32;
}

int uq_trellis_pack(const int32_t *states, int64_t nseq, int T, int L, int R, uint32_t *packed, void *stream) {
    const int64_t words = uq_trellis_packed_words(T, L, R);
    if (nseq < 0 || words == 0) return uq::fail(UQ_ERR_INVALID, "uq_trellis_pack: bad arguments (T=%d L=%d R=%d)", T, L, R);
    if (nseq == 0) return UQ_OK;
    if (!states || !packed) return uq::fail(UQ_ERR_INVALID, "uq_trellis_pack: null pointer");
    const int64_t n = nseq * words;
    const int grid = int(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, int64_t(uq::num_sms()) * 16)));
    { uq::ProfScope _p("pack", UQ_STREAM(stream)); pack_kernel<<<grid, 256, 0, UQ_STREAM(stream)>>>(states, nseq, T, L, R, int(words), packed); }
    return uq::check_cuda("pack_kernel launch");
}

int uq_trellis_unpack(const uint32_t *packed, int64_t nseq, int T, int L, int R, int32_t *states, void *stream) {
    const int64_t words = uq_trellis_packed_words(T, L, R);
    if (nseq < 0 || words == 0) return uq::fail(UQ_ERR_INVALID, "uq_trellis_unpack: bad arguments (T=%d L=%d R=%d)", T, L, R);
    if (nseq == 0) return UQ_OK;
    if (!states || !packed) return uq::fail(UQ_ERR_INVALID, "uq_trellis_unpack: null pointer");
    const int64_t n = nseq * T;
    const int grid = int(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, int64_t(uq::num_sms()) * 16)));
    { uq::ProfScope _p("unpack", UQ_STREAM(stream)); unpack_kernel<<<grid, 256, 0, UQ_STREAM(stream)>>>(packed, nseq, T, L, R, int(words), states); }
    return uq::check_cuda("unpack_kernel launch");
}

}  // extern "C"
