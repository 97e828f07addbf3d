// Importance-weighted quantization pipelines: the builders' recipe around the
// hot path (buildtrellis.py:16-20, buildalloc.py:21-24), fused on the device.
//
//   H' = max(H, max(H) * 1e-3), sH = sqrt(H'), A = W * sH        (fp64)
//   Arot = rht_rows(A)                                          (fp64 stages)
//   trellis: Ah_rot = trellis_quant_fast(Arot)  (float32 from here)
//   e8:      Ah_rot = q_e8_fast(Arot, fixed_step)               (fp64)
//   Ah = irht_rows(Ah_rot, n0);  What = float32(Ah / sH)
//   err = { sum (A - Ah)^2, sum A^2 }   (weighted NMSE = err[0] / err[1])
//
// Stages: column scale -> forward RHT (writes float32 for the trellis, since
// trellis_quant_fast starts with A.astype(float32)) -> group normalisation ->
// Viterbi + traceback -> decode -> inverse RHT with the /sH epilogue and the
// error partial sums.  Intermediates live in the caller's workspace.
#include <cuda_runtime.h>

#include <algorithm>

#include "uq_common.cuh"

namespace uq {
int rht_forward(const void *in, int in_dtype, int64_t rows, int64_t n0, int64_t ld_in, const double *colscale,
                const double *pre, const double *signs, void *out, int out_dtype, int64_t ld_out, cudaStream_t st);
int rht_inverse(const void *in, int in_dtype, int64_t rows, int64_t n, int64_t ld_in, int64_t n0,
                const double *signs, const double *colscale, const double *pre, void *out, int out_dtype,
                int64_t ld_out, const void *ref_w, int ref_dtype, int64_t ld_w, double *err_partial, double *err,
                cudaStream_t st);
int rht_prescale(const double *colscale, const double *signs, int64_t n0, int64_t n, double *pre, cudaStream_t st);
int64_t rht_tiles(int64_t rows, int64_t n);
int e8_quant(const void *A, int a_dtype, int64_t size, int64_t group, double step, double *rec, int16_t *idx,
             double *rms_out, cudaStream_t st);
size_t e8_search_ws_bytes(int64_t rows, int64_t n);
int e8_scale_search(const double *A, int64_t rows, int64_t n, double step, double *rec, int16_t *idx,
                    int32_t *choice_out, double *lam_host, void *ws, size_t ws_bytes, cudaStream_t st);
int trellis_normalize(const void *A, int dtype, int64_t nrow, int64_t T, int64_t lda, int64_t Tp, int64_t group,
                      float *xn, float *sc, cudaStream_t st);
size_t trellis_ws_bytes(int64_t nseq, int T, int L, int R);
int trellis_viterbi(const float *xn, int64_t nseq, int T, int L, int R, const float *cw, int32_t *states,
                    void *ws, size_t ws_bytes, cudaStream_t st);
int trellis_decode(const int32_t *states, const float *cw, const float *sc, int64_t group, int64_t ntot,
                   float *out, cudaStream_t st);
}  // namespace uq

namespace {

// sH[j] = sqrt(max(H[j], max(H) * 1e-3))  (one CTA; max is order independent)
__global__ void importance_scale_kernel(const double *H, int64_t n0, double *sH) {
    __shared__ double red[32];
    double mx = -INFINITY;
    for (int64_t j = threadIdx.x; j < n0; j += blockDim.x) mx = fmax(mx, H[j]);
    for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        mx = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
        for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (threadIdx.x == 0) red[0] = mx;
    }
    __syncthreads();
    const double floor_v = d_mul(red[0], 1e-3);
    for (int64_t j = threadIdx.x; j < n0; j += blockDim.x) sH[j] = sqrt(fmax(H[j], floor_v));
}

struct TrellisPlan {
    int64_t n, ntot, padded, nseq, ngroups, tiles;
    size_t vit_ws;
};

TrellisPlan plan_trellis(int64_t rows, int64_t n0, int L, int R, int seg, int group) {
    TrellisPlan p{};
    p.n = uq_next_pow2(n0);
    p.ntot = rows * p.n;
    p.padded = (p.ntot + group - 1) / group * group;
    p.nseq = seg > 0 ? p.padded / seg : 0;
    p.ngroups = p.padded / group;
    p.tiles = uq::rht_tiles(rows, p.n);
    p.vit_ws = uq::trellis_ws_bytes(p.nseq, seg, L, R);
    return p;
}

size_t carve_trellis(const TrellisPlan &p, int64_t n0, bool need_states, bool need_sc, void *base, double **sH,
                     double **pre, float **X, int32_t **states, float **sc, double **part, void **vit) {
    uq::Carver c(base, ~size_t(0));
    *sH = c.take<double>(size_t(n0));
    *pre = c.take<double>(size_t(p.n));
    *X = c.take<float>(size_t(p.padded));
    *states = need_states ? c.take<int32_t>(size_t(p.padded)) : nullptr;
    *sc = need_sc ? c.take<float>(size_t(p.ngroups)) : nullptr;
    *part = c.take<double>(size_t(2 * p.tiles));
    *vit = c.take<char>(p.vit_ws);
    return c.off;
}

int check_common(int64_t rows, int64_t n0, int64_t ldw, int w_dtype, int group, const char *who) {
    if (rows < 0 || n0 < 1 || ldw < n0 || !uq::dtype_size(w_dtype))
        return uq::fail(UQ_ERR_INVALID, "%s: bad shape (rows=%lld n0=%lld ldw=%lld)", who, (long long)rows,
                        (long long)n0, (long long)ldw);
    if (uq_next_pow2(n0) > 32768) return uq::fail(UQ_ERR_UNSUPPORTED, "%s: padded width > 32768 not built", who);
    if (group < 8 || group % 8 || group > 8192)
        return uq::fail(UQ_ERR_UNSUPPORTED, "%s: group %d must be a multiple of 8 in [8, 8192]", who, group);
    return UQ_OK;
}

}  // namespace

// ---- weighted NMSE (qlab.py:53-54) --------------------------------------------
// sum((A - Ah)^2) and sum(A^2) in fp64: fixed grid of CTAs, per-thread
// grid-stride sums, warp trees and a CTA tree into per-CTA partials, then one
// CTA sums the partials in index order -- deterministic for a given size.
constexpr int kNmseBlocks = 592;

template <typename TA, typename TB>
__global__ void wnmse_partial_kernel(const TA *A, const TB *Ah, int64_t n, double *part) {
    __shared__ double s0[32], s1[32];
    double e = 0.0, a2 = 0.0;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const double a = double(__ldg(A + i)), d = d_sub(a, double(__ldg(Ah + i)));
        e = d_add(e, d_mul(d, d));
        a2 = d_add(a2, d_mul(a, a));
    }
    for (int o = 16; o > 0; o >>= 1) {
        e = d_add(e, __shfl_xor_sync(0xffffffffu, e, o));
        a2 = d_add(a2, __shfl_xor_sync(0xffffffffu, a2, o));
    }
    if ((threadIdx.x & 31) == 0) { s0[threadIdx.x >> 5] = e; s1[threadIdx.x >> 5] = a2; }
    __syncthreads();
    if (threadIdx.x == 0) {
        double t0 = 0.0, t1 = 0.0;
        for (int w = 0; w < int(blockDim.x >> 5); ++w) { t0 = d_add(t0, s0[w]); t1 = d_add(t1, s1[w]); }
        part[2 * blockIdx.x] = t0;
        part[2 * blockIdx.x + 1] = t1;
    }
}

__global__ void wnmse_final_kernel(const double *part, int count, double *out) {
    if (threadIdx.x != 0) return;
    double t0 = 0.0, t1 = 0.0;
    for (int i = 0; i < count; ++i) { t0 = d_add(t0, part[2 * i]); t1 = d_add(t1, part[2 * i + 1]); }
    out[0] = t0;
    out[1] = t1;
}

extern "C" {
int uq_rht28_rows(const void *A, int a_dtype, int64_t rows, int64_t n0, int64_t lda, const double *colscale,
                  const double *signs, double *out, void *stream);
int uq_irht28_rows(const void *X, int x_dtype, int64_t rows, int64_t n0, int64_t ldx, const double *colscale,
                   const double *signs, void *out, int out_dtype, int64_t ld_out, void *stream);

size_t uq_quant_trellis_workspace_bytes(int64_t rows, int64_t n0, int L, int R, int seg, int group) {
    if (rows < 0 || n0 < 1 || seg < 1 || group < 8) return 0;
    const TrellisPlan p = plan_trellis(rows, n0, L, R, seg, group);
    double *a, *a2; float *b; int32_t *c; float *d; double *e; void *f;
    return carve_trellis(p, n0, true, true, nullptr, &a, &a2, &b, &c, &d, &e, &f);
}

int uq_quant_trellis(const void *W, int w_dtype, int64_t rows, int64_t n0, int64_t ldw, const double *H, int L,
                     int R, int seg, int group, const double *signs, const float *cw, float *What, int32_t *states,
                     float *sc, double *err, void *workspace, size_t workspace_bytes, void *stream) {
    uq::NvtxRange _r("uq_quant_trellis");
    int rc = check_common(rows, n0, ldw, w_dtype, group, "uq_quant_trellis");
    if (rc) return rc;
    if (R < 1 || R > 4 || L < 6 || L > 16 || L < 2 * R || seg < 1)
        return uq::fail(UQ_ERR_UNSUPPORTED, "uq_quant_trellis: (L=%d, R=%d, seg=%d) not built", L, R, seg);
    if (rows == 0) return UQ_OK;
    if (!W || !H || !signs || !cw || !What || !workspace) return uq::fail(UQ_ERR_INVALID, "uq_quant_trellis: null pointer");
    const TrellisPlan p = plan_trellis(rows, n0, L, R, seg, group);
    if (p.padded % seg) return uq::fail(UQ_ERR_INVALID, "uq_quant_trellis: padded size %lld not divisible by seg %d",
                                        (long long)p.padded, seg);
    double *sH, *pre, *part;
    float *X, *scw;
    int32_t *stw;
    void *vit;
    const size_t need = carve_trellis(p, n0, states == nullptr, sc == nullptr, workspace, &sH, &pre, &X, &stw, &scw,
                                      &part, &vit);
    if (workspace_bytes < need) return uq::fail(UQ_ERR_WORKSPACE, "uq_quant_trellis: workspace %zu < %zu", workspace_bytes, need);
    if (!states) states = stw;
    if (!sc) sc = scw;
    cudaStream_t st = UQ_STREAM(stream);
    { uq::ProfScope _p("importance_scale", st); importance_scale_kernel<<<1, 1024, 0, st>>>(H, n0, sH); }
    if ((rc = uq::check_cuda("importance_scale_kernel launch"))) return rc;
    if ((rc = uq::rht_prescale(sH, signs, n0, p.n, pre, st))) return rc;
    // A = W * sH, rotated, rounded to float32 (trellis_quant_fast: A.astype(float32))
    if ((rc = uq::rht_forward(W, w_dtype, rows, n0, ldw, sH, pre, signs, X, UQ_F32, p.n, st))) return rc;
    if (p.padded > p.ntot) cudaMemsetAsync(X + p.ntot, 0, size_t(p.padded - p.ntot) * sizeof(float), st);
    if ((rc = uq::trellis_normalize(X, UQ_F32, 1, p.ntot, p.ntot, p.padded, group, X, sc, st))) return rc;
    if ((rc = uq::trellis_viterbi(X, p.nseq, seg, L, R, cw, states, vit, p.vit_ws, st))) return rc;
    if ((rc = uq::trellis_decode(states, cw, sc, group, p.ntot, X, st))) return rc;
    return uq::rht_inverse(X, UQ_F32, rows, p.n, p.n, n0, signs, sH, pre, What, UQ_F32, n0, W, w_dtype, ldw, part,
                           err, st);
}

size_t uq_quant_e8_workspace_bytes(int64_t rows, int64_t n0, int group) {
    if (rows < 0 || n0 < 1 || group < 8) return 0;
    const int64_t n = uq_next_pow2(n0);
    uq::Carver c(nullptr, ~size_t(0));
    c.take<double>(size_t(n0));
    c.take<double>(size_t(n));
    c.take<double>(size_t(rows * n));
    c.take<double>(size_t(2 * uq::rht_tiles(rows, n)));
    return c.off;
}

int uq_quant_e8(const void *W, int w_dtype, int64_t rows, int64_t n0, int64_t ldw, const double *H, double step,
                int group, const double *signs, float *What, int16_t *idx, double *err, void *workspace,
                size_t workspace_bytes, void *stream) {
    uq::NvtxRange _r("uq_quant_e8");
    int rc = check_common(rows, n0, ldw, w_dtype, group, "uq_quant_e8");
    if (rc) return rc;
    if (rows == 0) return UQ_OK;
    if (!W || !H || !signs || !What || !workspace) return uq::fail(UQ_ERR_INVALID, "uq_quant_e8: null pointer");
    const int64_t n = uq_next_pow2(n0);
    uq::Carver c(workspace, workspace_bytes);
    double *sH = c.take<double>(size_t(n0));
    double *pre = c.take<double>(size_t(n));
    double *X = c.take<double>(size_t(rows * n));
    double *part = c.take<double>(size_t(2 * uq::rht_tiles(rows, n)));
    if (!c.ok()) return uq::fail(UQ_ERR_WORKSPACE, "uq_quant_e8: workspace %zu < %zu", workspace_bytes, c.off);
    cudaStream_t st = UQ_STREAM(stream);
    { uq::ProfScope _p("importance_scale", st); importance_scale_kernel<<<1, 1024, 0, st>>>(H, n0, sH); }
    if ((rc = uq::check_cuda("importance_scale_kernel launch"))) return rc;
    if ((rc = uq::rht_prescale(sH, signs, n0, n, pre, st))) return rc;
    if ((rc = uq::rht_forward(W, w_dtype, rows, n0, ldw, sH, pre, signs, X, UQ_F64, n, st))) return rc;
    if ((rc = uq::e8_quant(X, UQ_F64, rows * n, group, step, X, idx, nullptr, st))) return rc;
    return uq::rht_inverse(X, UQ_F64, rows, n, n, n0, signs, sH, pre, What, UQ_F32, n0, W, w_dtype, ldw, part, err,
                           st);
}

// Opt-in: the buildalloc recipe with the per-row scale search over 16
// candidate steps (uq_e8_scale_search) in place of the single fixed step.
size_t uq_quant_e8_search_workspace_bytes(int64_t rows, int64_t n0) {
    if (rows < 0 || n0 < 1) return 0;
    const int64_t n = uq_next_pow2(n0);
    if (n < 256) return 0;
    uq::Carver c(nullptr, ~size_t(0));
    c.take<double>(size_t(n0));
    c.take<double>(size_t(n));
    c.take<double>(size_t(rows * n));
    c.take<double>(size_t(2 * uq::rht_tiles(rows, n)));
    c.take<char>(uq::e8_search_ws_bytes(rows, n));
    return c.off;
}

int uq_quant_e8_search(const void *W, int w_dtype, int64_t rows, int64_t n0, int64_t ldw, const double *H,
                       double step, const double *signs, float *What, int16_t *idx, int32_t *choice,
                       double *lam_host, double *err, void *workspace, size_t workspace_bytes, void *stream) {
    uq::NvtxRange _r("uq_quant_e8_search");
    int rc = check_common(rows, n0, ldw, w_dtype, 256, "uq_quant_e8_search");
    if (rc) return rc;
    const int64_t n = uq_next_pow2(n0);
    if (n < 256) return uq::fail(UQ_ERR_INVALID, "uq_quant_e8_search: padded width %lld below one group", (long long)n);
    if (!(step > 0.0)) return uq::fail(UQ_ERR_INVALID, "uq_quant_e8_search: step must be > 0");
    if (rows == 0) {
        if (lam_host) *lam_host = 0.0;
        return UQ_OK;
    }
    if (!W || !H || !signs || !What || !workspace) return uq::fail(UQ_ERR_INVALID, "uq_quant_e8_search: null pointer");
    uq::Carver c(workspace, workspace_bytes);
    double *sH = c.take<double>(size_t(n0));
    double *pre = c.take<double>(size_t(n));
    double *X = c.take<double>(size_t(rows * n));
    double *part = c.take<double>(size_t(2 * uq::rht_tiles(rows, n)));
    const size_t sws = uq::e8_search_ws_bytes(rows, n);
    void *swsp = c.take<char>(sws);
    if (!c.ok()) return uq::fail(UQ_ERR_WORKSPACE, "uq_quant_e8_search: workspace %zu < %zu", workspace_bytes, c.off);
    cudaStream_t st = UQ_STREAM(stream);
    { uq::ProfScope _p("importance_scale", st); importance_scale_kernel<<<1, 1024, 0, st>>>(H, n0, sH); }
    if ((rc = uq::check_cuda("importance_scale_kernel launch"))) return rc;
    if ((rc = uq::rht_prescale(sH, signs, n0, n, pre, st))) return rc;
    if ((rc = uq::rht_forward(W, w_dtype, rows, n0, ldw, sH, pre, signs, X, UQ_F64, n, st))) return rc;
    if ((rc = uq::e8_scale_search(X, rows, n, step, X, idx, choice, lam_host, swsp, sws, st))) return rc;
    return uq::rht_inverse(X, UQ_F64, rows, n, n, n0, signs, sH, pre, What, UQ_F32, n0, W, w_dtype, ldw, part, err,
                           st);
}

size_t uq_wnmse_workspace_bytes(void) { return size_t(2) * kNmseBlocks * sizeof(double); }

int uq_wnmse_sums(const void *A, int a_dtype, const void *Ah, int ah_dtype, int64_t n, double *out2,
                  void *workspace, size_t workspace_bytes, void *stream) {
    if (n < 0 || !uq::dtype_size(a_dtype) || !uq::dtype_size(ah_dtype))
        return uq::fail(UQ_ERR_INVALID, "uq_wnmse_sums: bad arguments (n=%lld)", (long long)n);
    if (!out2) return uq::fail(UQ_ERR_INVALID, "uq_wnmse_sums: null output");
    if (!workspace || workspace_bytes < uq_wnmse_workspace_bytes())
        return uq::fail(UQ_ERR_WORKSPACE, "uq_wnmse_sums: workspace %zu < %zu bytes", workspace_bytes,
                        uq_wnmse_workspace_bytes());
    if (n > 0 && (!A || !Ah)) return uq::fail(UQ_ERR_INVALID, "uq_wnmse_sums: null input");
    const cudaStream_t st = UQ_STREAM(stream);
    double *part = static_cast<double *>(workspace);
    {
        uq::ProfScope _p("wnmse", st);
        const bool a64 = a_dtype == UQ_F64, b64 = ah_dtype == UQ_F64;
        if (a64 && b64) wnmse_partial_kernel<double, double><<<kNmseBlocks, 256, 0, st>>>(
            static_cast<const double *>(A), static_cast<const double *>(Ah), n, part);
        else if (a64) wnmse_partial_kernel<double, float><<<kNmseBlocks, 256, 0, st>>>(
            static_cast<const double *>(A), static_cast<const float *>(Ah), n, part);
        else if (b64) wnmse_partial_kernel<float, double><<<kNmseBlocks, 256, 0, st>>>(
            static_cast<const float *>(A), static_cast<const double *>(Ah), n, part);
        else wnmse_partial_kernel<float, float><<<kNmseBlocks, 256, 0, st>>>(
            static_cast<const float *>(A), static_cast<const float *>(Ah), n, part);
        wnmse_final_kernel<<<1, 32, 0, st>>>(part, kNmseBlocks, out2);
    }
    return uq::check_cuda("wnmse kernels launch");
}

// Opt-in: the buildalloc recipe with the block-factorised transform for
// n0 = 28 x 512 / 28 x 1024 (no padding).  Weighted error sums are taken in the
// rotated domain (the transform is orthogonal: equal to the original-domain
// sums up to rounding).
size_t uq_quant_e8_b28_workspace_bytes(int64_t rows, int64_t n0) {
    if (rows < 0 || n0 < 1) return 0;
    uq::Carver c(nullptr, ~size_t(0));
    c.take<double>(size_t(n0));
    c.take<double>(size_t(rows * n0));
    c.take<double>(size_t(rows * n0));
    c.take<unsigned char>(uq_wnmse_workspace_bytes());
    return c.off;
}

int uq_quant_e8_b28(const void *W, int w_dtype, int64_t rows, int64_t n0, int64_t ldw, const double *H, double step,
                    const double *signs, float *What, int16_t *idx, double *err, void *workspace,
                    size_t workspace_bytes, void *stream) {
    uq::NvtxRange _r("uq_quant_e8_b28");
    int rc = check_common(rows, n0, ldw, w_dtype, 256, "uq_quant_e8_b28");
    if (rc) return rc;
    if (n0 != 28 * 512 && n0 != 28 * 1024)
        return uq::fail(UQ_ERR_INVALID, "uq_quant_e8_b28: n0 = %lld is not 28 x 512 or 28 x 1024", (long long)n0);
    if (rows == 0) return UQ_OK;
    if (!W || !H || !signs || !What || !err || !workspace) return uq::fail(UQ_ERR_INVALID, "uq_quant_e8_b28: null pointer");
    uq::Carver c(workspace, workspace_bytes);
    double *sH = c.take<double>(size_t(n0));
    double *X = c.take<double>(size_t(rows * n0));
    double *Xq = c.take<double>(size_t(rows * n0));
    unsigned char *part = c.take<unsigned char>(uq_wnmse_workspace_bytes());
    if (!c.ok()) return uq::fail(UQ_ERR_WORKSPACE, "uq_quant_e8_b28: workspace %zu < %zu", workspace_bytes, c.off);
    cudaStream_t st = UQ_STREAM(stream);
    { uq::ProfScope _p("importance_scale", st); importance_scale_kernel<<<1, 1024, 0, st>>>(H, n0, sH); }
    if ((rc = uq::check_cuda("importance_scale_kernel launch"))) return rc;
    if ((rc = uq_rht28_rows(W, w_dtype, rows, n0, ldw, sH, signs, X, stream))) return rc;
    if ((rc = uq::e8_quant(X, UQ_F64, rows * n0, 256, step, Xq, idx, nullptr, st))) return rc;
    if ((rc = uq_wnmse_sums(X, UQ_F64, Xq, UQ_F64, rows * n0, err, part, uq_wnmse_workspace_bytes(), stream))) return rc;
    return uq_irht28_rows(Xq, UQ_F64, rows, n0, n0, sH, signs, What, UQ_F32, n0, stream);
}

}  // extern "C"
