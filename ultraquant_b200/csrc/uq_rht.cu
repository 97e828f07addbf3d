// Randomized Hadamard transform along rows (qlab.py:66-98) for sm_100a.
//
// Bit-exactness: the reference runs the Sylvester butterflies in fp64 with
// stage order h = 1, 2, 4, ..., n/2.  Every output is the same sequence of
// correctly rounded adds / subtracts whatever the data layout, so the kernel
// only has to keep the stage order.  Scaling uses IEEE division by sqrt(n)
// (forward) and by n (inverse) exactly like numpy.
//
// Layout: a CTA owns a tile of 2^NB consecutive elements (NB = max(12, b),
// n = 2^b; one tile holds 2^(NB-b) rows).  The tile lives in shared memory as
// fp64 with the XOR swizzle P(E) = E ^ ((E >> 4) & 15) on the element index,
// which makes every access pattern below bank-conflict free.  Each of the
// 2^(NB-4) threads holds 16 elements in registers per pass; pass p keeps the
// index bits [p, p+4) in registers and runs the stages of those bits.  The
// final pass (p = NB-4) has consecutive threads on consecutive elements, so
// the global store is coalesced; the load is coalesced the same way.
#include <cuda_runtime.h>

#include "uq_common.cuh"

namespace {

constexpr int kMaxBits = 14;  // n <= 16384 doubles = 128 KB of shared memory per CTA

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
    void *out;
    int64_t ld_out, ncols_out;   // output row stride, columns written (< n crops)
    double sqrt_n, n_d;
    // optional error statistics for the inverse of the importance pipeline:
    // A = rn(W * colscale) recomputed from W, partial sums per CTA.
    const void *ref_w;           // W (rows, n0) with stride ld_w, dtype = ref_dtype
    int64_t ld_w;
    int ref_dtype;
    double *err_partial;         // [gridDim.x * 2]
};

template <typename TIn, typename TOut, int MODE, int MAXT>
__global__ void __launch_bounds__(MAXT)
rht_tile_kernel(RhtArgs a) {
    extern __shared__ double tile[];
    const int b = a.b;
    const int NB = b > 12 ? b : 12;
    const int nthr = 1 << (NB - 4);
    const int tid = threadIdx.x;
    const int64_t n = int64_t(1) << b;
    const int rows_per_tile = 1 << (NB - b);
    const int64_t row0 = int64_t(blockIdx.x) * rows_per_tile;
    const TIn *in = static_cast<const TIn *>(a.in);

    // ---- coalesced load: combined index E = tid + nthr * j ------------------
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int E = tid + nthr * j;
        const int64_t r = row0 + (E >> b);
        const int e = E & int(n - 1);
        double x;
        if (MODE == MODE_FWD) {
            double av = 0.0;
            if (r < a.rows && e < a.n0) {
                av = ld_as_f64(in + r * a.ld_in + e);
                if (a.colscale) av = d_mul(av, __ldg(a.colscale + e));
            }
            x = d_mul(av, __ldg(a.signs + e));
        } else {
            x = 0.0;
            if (r < a.rows) x = d_mul(ld_as_f64(in + r * a.ld_in + e), a.sqrt_n);
        }
        tile[swz(E)] = x;
    }
    __syncthreads();

    // ---- passes: bits [p, p+4) in registers --------------------------------
    int done = 0;  // stages (index bits) already applied
    const int last_p = NB - 4;
    for (int p = 0;; p += 4) {
        if (p > last_p) p = last_p;
        const int base = (tid & ((1 << p) - 1)) | ((tid >> p) << (p + 4));
        double x[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] = tile[swz(base + (j << p))];
        const int hi = (p + 4 < b) ? p + 4 : b;
        const int lo = done > p ? done : p;
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
        if (hi > done) done = hi;
        if (p == last_p) {
            // ---- epilogue: scale and store (coalesced: base == tid) --------
            double se = 0.0, sa = 0.0;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int E = base + (j << p);
                const int64_t r = row0 + (E >> b);
                const int e = E & int(n - 1);
                if (r >= a.rows || e >= a.ncols_out) continue;
                double y;
                if (MODE == MODE_FWD) {
                    y = x[j] / a.sqrt_n;
                } else {
                    y = d_mul(x[j] / a.n_d, __ldg(a.signs + e));
                    if (a.err_partial) {
                        double w = a.ref_dtype == UQ_F32
                            ? double(__ldg(static_cast<const float *>(a.ref_w) + r * a.ld_w + e))
                            : __ldg(static_cast<const double *>(a.ref_w) + r * a.ld_w + e);
                        const double A = d_mul(w, __ldg(a.colscale + e));
                        const double dd = d_sub(A, y);
                        se = d_add(se, d_mul(dd, dd));
                        sa = d_add(sa, d_mul(A, A));
                    }
                    if (a.colscale) y = y / __ldg(a.colscale + e);
                }
                static_cast<TOut *>(a.out)[r * a.ld_out + e] = TOut(y);
            }
            if (MODE == MODE_INV && a.err_partial) {
                // deterministic CTA reduction: warp tree, then warp 0
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
                    a.err_partial[2 * blockIdx.x] = s0;
                    a.err_partial[2 * blockIdx.x + 1] = s1;
                }
            }
            break;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) tile[swz(base + (j << p))] = x[j];
        __syncthreads();
    }
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

template <typename TIn, typename TOut, int MODE>
int launch_rht(const RhtArgs &a, cudaStream_t st) {
    const int NB = a.b > 12 ? a.b : 12;
    const int nthr = 1 << (NB - 4);
    const int rows_per_tile = 1 << (NB - a.b);
    const int64_t grid = (a.rows + rows_per_tile - 1) / rows_per_tile;
    const size_t smem = sizeof(double) << NB;
    // 16 fp64 values per thread: keep the 128-register budget for tiles up to
    // 2^13 elements; 2^14-element tiles need 1024 threads (64 registers).
    auto kern = nthr <= 512 ? rht_tile_kernel<TIn, TOut, MODE, 512> : rht_tile_kernel<TIn, TOut, MODE, 1024>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
        return uq::check_cuda("rht: set smem attribute");
    if (grid > 0) { uq::ProfScope _p("rht", st); kern<<<unsigned(grid), nthr, smem, st>>>(a); }
    return uq::check_cuda("rht_tile_kernel launch");
}

}  // namespace

namespace uq {

// Forward RHT with optional column pre-scale; output fp64 or fp32.
int rht_forward(const void *in, int in_dtype, int64_t rows, int64_t n0, int64_t ld_in,
                const double *colscale, const double *signs, void *out, int out_dtype,
                int64_t ld_out, cudaStream_t st) {
    RhtArgs a{};
    a.in = in; a.rows = rows; a.n0 = n0; a.ld_in = ld_in;
    const int64_t n = uq_next_pow2(n0);
    a.b = ilog2(n);
    a.signs = signs; a.colscale = colscale; a.out = out;
    a.ld_out = ld_out; a.ncols_out = n;
    a.sqrt_n = sqrt(double(n)); a.n_d = double(n);
    if (a.b > kMaxBits) return fail(UQ_ERR_UNSUPPORTED, "rht: n = %lld > 16384 not built", (long long)n);
    if (in_dtype == UQ_F64 && out_dtype == UQ_F64) return launch_rht<double, double, MODE_FWD>(a, st);
    if (in_dtype == UQ_F32 && out_dtype == UQ_F64) return launch_rht<float, double, MODE_FWD>(a, st);
    if (in_dtype == UQ_F64 && out_dtype == UQ_F32) return launch_rht<double, float, MODE_FWD>(a, st);
    if (in_dtype == UQ_F32 && out_dtype == UQ_F32) return launch_rht<float, float, MODE_FWD>(a, st);
    return fail(UQ_ERR_INVALID, "rht: bad dtype");
}

// Inverse RHT with optional column post-division and error statistics.
int rht_inverse(const void *in, int in_dtype, int64_t rows, int64_t n, int64_t ld_in,
                int64_t n0, const double *signs, const double *colscale, void *out,
                int out_dtype, int64_t ld_out, const void *ref_w, int ref_dtype,
                int64_t ld_w, double *err_partial, double *err, cudaStream_t st) {
    RhtArgs a{};
    a.in = in; a.rows = rows; a.n0 = n; a.ld_in = ld_in;
    a.b = ilog2(n);
    a.signs = signs; a.colscale = colscale; a.out = out;
    a.ld_out = ld_out; a.ncols_out = n0;
    a.sqrt_n = sqrt(double(n)); a.n_d = double(n);
    a.ref_w = ref_w; a.ref_dtype = ref_dtype; a.ld_w = ld_w; a.err_partial = err ? err_partial : nullptr;
    if (a.b > kMaxBits) return fail(UQ_ERR_UNSUPPORTED, "irht: n = %lld > 16384 not built", (long long)n);
    int rc;
    if (in_dtype == UQ_F64 && out_dtype == UQ_F64) rc = launch_rht<double, double, MODE_INV>(a, st);
    else if (in_dtype == UQ_F32 && out_dtype == UQ_F64) rc = launch_rht<float, double, MODE_INV>(a, st);
    else if (in_dtype == UQ_F64 && out_dtype == UQ_F32) rc = launch_rht<double, float, MODE_INV>(a, st);
    else if (in_dtype == UQ_F32 && out_dtype == UQ_F32) rc = launch_rht<float, float, MODE_INV>(a, st);
    else return fail(UQ_ERR_INVALID, "irht: bad dtype");
    if (rc != UQ_OK || !err) return rc;
    const int NB = a.b > 12 ? a.b : 12;
    const int64_t tiles = (rows + (1 << (NB - a.b)) - 1) >> (NB - a.b);
    { uq::ProfScope _p("sum_pairs", st); sum_pairs_kernel<<<1, 256, 0, st>>>(err_partial, tiles, err); }
    return check_cuda("sum_pairs_kernel launch");
}

int64_t rht_tiles(int64_t rows, int64_t n) {
    const int b = ilog2(n);
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
    return uq::rht_forward(A, a_dtype, rows, n0, lda, nullptr, signs, out, UQ_F64, n, UQ_STREAM(stream));
}

int uq_irht_rows(const void *X, int x_dtype, int64_t rows, int64_t n, int64_t ldx, int64_t n0,
                 const double *signs, double *out, void *stream) {
    if (rows < 0 || !uq::is_pow2(n) || ldx < n || n0 < 0 || n0 > n || !uq::dtype_size(x_dtype))
        return uq::fail(UQ_ERR_INVALID, "uq_irht_rows: bad shape (rows=%lld n=%lld n0=%lld)",
                        (long long)rows, (long long)n, (long long)n0);
    if (rows == 0 || n0 == 0) return UQ_OK;
    if (!X || !signs || !out) return uq::fail(UQ_ERR_INVALID, "uq_irht_rows: null pointer");
    return uq::rht_inverse(X, x_dtype, rows, n, ldx, n0, signs, nullptr, out, UQ_F64, n0,
                           nullptr, 0, 0, nullptr, nullptr, UQ_STREAM(stream));
}

}  // extern "C"
