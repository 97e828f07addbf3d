/*
 * uq_b200.h -- C ABI of the B200 (sm_100a) quantization hot path:
 * randomized Hadamard transform, E8 nearest-point quantizer and the
 * bitshift-trellis Viterbi encoder / decoder of UltraQuant.
 *
 * The reference exposes this path as plain Python module functions on numpy
 * arrays (qlab.py, trellis.py, qat.py).  Each entry point below names the
 * reference function it replaces.  The Python package ``ultraquant_b200``
 * wraps these calls in the reference's exact signatures through ctypes.
 *
 * Conventions
 *  - All array pointers are DEVICE pointers unless the name ends in _host.
 *  - Row-major layouts, explicit leading dimensions (in elements).
 *  - ``stream`` is a cudaStream_t passed as void* (NULL = legacy default).
 *  - Every entry point returns a uq_status; on failure uq_last_error()
 *    returns a message for the calling thread.  No entry point has a CPU
 *    fallback.
 *  - Entry points never synchronise the stream unless documented (the E8
 *    calibration reads scalar results back to the host).
 *  - dtype codes: UQ_F32 = 0, UQ_F64 = 1.
 */
#ifndef UQ_B200_H
#define UQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum uq_status {
    UQ_OK = 0,
    UQ_ERR_INVALID = 1,      /* bad shape / argument (reference: numpy ValueError) */
    UQ_ERR_UNSUPPORTED = 2,  /* valid for the reference but not built here (e.g. L > 16) */
    UQ_ERR_CUDA = 3,         /* CUDA runtime / launch error */
    UQ_ERR_WORKSPACE = 4,    /* workspace smaller than the *_workspace_bytes() query */
    UQ_ERR_TIMEOUT = 5       /* a device wait exceeded its bound */
};

enum uq_dtype { UQ_F32 = 0, UQ_F64 = 1 };

int uq_version(void);
const char *uq_status_string(int status);
const char *uq_last_error(void);

/* ---------------------------------------------------------------------
 * Randomized Hadamard transform (qlab.py:66-98)
 * ------------------------------------------------------------------- */

/* qlab.py:78, :96 -- ``np.random.RandomState(seed).choice([-1., 1.], n)``:
 * legacy MT19937, one 32-bit draw per sign, bit 0 selects +1.  Host output. */
int uq_rht_signs(uint32_t seed, int64_t n, double *out_host);

/* qlab.py:66-69 -- next power of two >= n0. */
int64_t uq_next_pow2(int64_t n0);

/* qlab.py:71-85 rht_rows(A, seed): out[rows, n] = FWHT(pad(A) * d) / sqrt(n),
 * fp64, stages h = 1..n/2 in order (bit-exact with numpy).  A is f32 or f64
 * (a_dtype), row stride lda >= n0.  signs: device, length n = next_pow2(n0).
 * n <= 32768 (larger n returns UQ_ERR_UNSUPPORTED). */
int uq_rht_rows(const void *A, int a_dtype, int64_t rows, int64_t n0, int64_t lda,
                const double *signs, double *out, void *stream);

/* qlab.py:87-98 irht_rows(X, n0, seed): out[rows, n0] =
 * (FWHT(X * sqrt(n)) / n * d)[:, :n0], fp64 (a float32 X is widened exactly,
 * as numpy 2 promotes it).  X has n (power of two) columns, stride ldx. */
int uq_irht_rows(const void *X, int x_dtype, int64_t rows, int64_t n, int64_t ldx,
                 int64_t n0, const double *signs, double *out, void *stream);

/* ---------------------------------------------------------------------
 * E8 lattice (qlab.py:133-183)
 * ------------------------------------------------------------------- */

/* Opt-in block-factorised transform for n0 = 28 x 512 or 28 x 1024 (the
 * ffn_down widths 14336 / 28672 without padding); no counterpart in the
 * reference, which pads to a power of two (qlab.py:75-77).  Forward:
 * (H_28 (x) H_P) D (A * colscale) * RN(1/sqrt(n0)) with H_28 the Paley
 * Hadamard matrix of order 28, D the RandomState(seed) signs of length n0
 * (`signs`), colscale nullable; out (rows, n0) fp64.  Inverse: the transpose,
 * then * d, or / (colscale * d) when colscale is given; out float32 or fp64
 * with row stride ld_out.  Operation order: oracle rht28_rows / irht28_rows. */
int uq_rht28_rows(const void *A, int a_dtype, int64_t rows, int64_t n0, int64_t lda,
                  const double *colscale, const double *signs, double *out, void *stream);
int uq_irht28_rows(const void *X, int x_dtype, int64_t rows, int64_t n0, int64_t ldx,
                   const double *colscale, const double *signs, void *out, int out_dtype,
                   int64_t ld_out, void *stream);

/* qlab.py:100-106 q_uniform(A, bpw, bs): per block of bs values, amax =
 * max|x| + 1e-12, out = rint(x / amax * lvl) / lvl * amax in the array's
 * dtype (UQ_F32 / UQ_F64); lvl = 2^(round(bpw) - 1) - 1 computed by the
 * caller (Python round).  size must be a multiple of bs. */
int uq_q_uniform(const void *A, int dtype, int64_t size, int64_t bs, int64_t lvl, void *out,
                 void *stream);

/* qlab.py:185-198 q_e8(A, bpw, group_scale): finite-codebook E8 quantizer.
 * A: `size` values (UQ_F32 / UQ_F64), flattened and zero-padded to whole
 * groups of `group` (a multiple of 8, at most 8192); s = sqrt(mean(g^2)) +
 * 1e-12 per group, gn = g / s as 8-vectors, out[e] = cb[nearest] * s (fp64,
 * `size` values).  cb: K x 8 fp64 codewords, cb32 the same rounded to fp32
 * (16-byte aligned).  When cb is qlab.py:111-124's e8_codebook(K) -- the K
 * grid points of smallest norm, divided by `scale` -- pass that scale and
 * norm_cut = the K-th smallest lattice norm (+inf when K covers the grid),
 * which lets vectors whose nearest lattice point is a codeword skip the
 * search; pass norm_cut = 0 for any other codebook.  Nearest = smallest
 * Euclidean distance (cKDTree.query); on an exact fp64 tie the lowest index.
 * Synchronises the stream; a non-finite gn returns UQ_ERR_INVALID (cKDTree's
 * ValueError).  Workspace: uq_q_e8_workspace_bytes(size, group). */
size_t uq_q_e8_workspace_bytes(int64_t size, int64_t group);
int uq_q_e8(const void *A, int a_dtype, int64_t size, int64_t group, const double *cb,
            const float *cb32, int64_t K, double scale, double norm_cut, double *out,
            void *workspace, size_t workspace_bytes, void *stream);

/* qlab.py:133-142 _d8_decode(Y): Y, out are (nvec, 8) fp64. */
int uq_d8_decode(const double *Y, int64_t nvec, double *out, void *stream);

/* qlab.py:144-149 e8_decode(Y): nearest point of D8 u (D8 + 1/2). */
int uq_e8_decode(const double *Y, int64_t nvec, double *out, void *stream);

/* qlab.py:159-170, 181-183 q_e8_fast(A, group=group, fixed_step=step) and the
 * calibrated form once its step is known: per-group RMS (numpy pairwise
 * order) + 1e-12, gn = g / rms, pts = e8_decode(gn / step),
 * rec = pts * step * rms, flattened A of `size` elements (zero-padded to the
 * group).  rec: `size` fp64.  idx (nullable): 2*pts as int16, size rounded up
 * to a multiple of 8. */
int uq_e8_quant(const void *A, int a_dtype, int64_t size, int64_t group, double step,
                double *rec, int16_t *idx, void *stream);

/* qlab.py:151-156 _entropy_bpw(pts): entropy of the distinct 8-tuples
 * (2*pts truncated to int64) / 8.  pts: (nvec, 8) fp64; result written to
 * bpw (device, one fp64).  Needs uq_e8_entropy_workspace_bytes(nvec). */
size_t uq_e8_entropy_workspace_bytes(int64_t nvec);
int uq_e8_entropy_bpw(const double *pts, int64_t nvec, double *bpw, void *workspace,
                      size_t workspace_bytes, void *stream);

/* qlab.py:171-180 -- calibrated step of q_e8_fast(A, target_bpw, group):
 * 600k-vector MT19937 subsample (RandomState(0).randint), 18 bisection steps
 * on [0.3, 10] of the entropy rate.  Synchronises `stream`; the step is
 * written to *step_host. */
size_t uq_e8_calibrate_workspace_bytes(int64_t size, int64_t group);
int uq_e8_calibrate(const void *A, int a_dtype, int64_t size, int64_t group,
                    double target_bpw, double *step_host, void *workspace,
                    size_t workspace_bytes, void *stream);

/* The pieces of uq_e8_calibrate, for a tensor whose row blocks live on
 * several devices (the sample spans the whole tensor):
 *  - uq_e8_sample_indices: qlab.py:173's RandomState(0).randint(0, nvec, ns)
 *    (host memory, no device work);
 *  - uq_e8_sample_gn: out[i] = the normalised 8-vector gn (qlab.py:167-168:
 *    x / (sqrt(mean(g^2)) + 1e-12) of its group) of local vector vec_ids[i]
 *    (device array) of A, a block of whole groups of the tensor;
 *  - uq_e8_calibrate_sample: the 18-step bisection (qlab.py:174-180) on ns
 *    such vectors in sample order; synchronises, step in *step_host. */
int uq_e8_sample_indices(int64_t nvec, int64_t ns, int64_t *out_host);
size_t uq_e8_sample_gn_workspace_bytes(int64_t size, int64_t group);
int uq_e8_sample_gn(const void *A, int a_dtype, int64_t size, int64_t group, const int64_t *vec_ids,
                    int64_t count, double *out, void *workspace, size_t workspace_bytes, void *stream);
size_t uq_e8_calibrate_sample_workspace_bytes(int64_t ns);
int uq_e8_calibrate_sample(const double *sub, int64_t ns, double target_bpw, double *step_host,
                           void *workspace, size_t workspace_bytes, void *stream);

/* Opt-in per-row scale search over 16 candidate steps (no counterpart in the
 * reference, whose q_e8_fast uses one global step, qlab.py:159-183).  A:
 * rotated matrix (rows, n) fp64, 16-byte aligned, n a multiple of 256 in
 * [256, 2^17]; groups of 256.  Candidates step_c = step * 2^((c - 8) / 8),
 * c = 0..15.  For each row and candidate: D = sum (A - rec)^2 (numpy order)
 * and H = the bits of the row's lattice coordinates z = 2p under their own
 * histogram.  Row r takes the first argmin of D + lam * H at the smallest
 * lam whose total H does not exceed the global step's (c = 8).  Outputs
 * (nullable): rec (rows * n, may equal A), idx = 2p int16, choice (rows)
 * int32 candidate per row, *lam_host.  Synchronises the stream (lam is
 * chosen on the host).  UQ_ERR_UNSUPPORTED if some |2p| exceeds 255, or
 * for more than (2^31 - 1) / 16 rows (one CTA per row and candidate). */
size_t uq_e8_scale_search_workspace_bytes(int64_t rows, int64_t n);
int uq_e8_scale_search(const double *A, int64_t rows, int64_t n, double step, double *rec, int16_t *idx,
                       int32_t *choice, double *lam_host, void *workspace, size_t workspace_bytes,
                       void *stream);

/* ---------------------------------------------------------------------
 * Bitshift trellis (trellis.py:14-108, qat.py:11-59)
 * ------------------------------------------------------------------- */

/* trellis.py:14-19 codebook(L): hashed state -> u -> inverse normal CDF
 * (Wichura AS241 in fp64) -> float32.  out: 2^L floats, 1 <= L <= 16. */
int uq_trellis_codebook(int L, float *out, void *stream);

/* trellis.py:69-80 (= qat.py:135-138): flatten `ntot` values (f32 or f64,
 * rounded to f32), zero-pad to a multiple of `group`, sc[g] = sqrt(mean(g^2))
 * + 1e-12 in float32 (numpy pairwise order), xn = g / sc.  The padded length
 * must be a multiple of `seg` (else UQ_ERR_INVALID, as numpy's reshape
 * fails).  xn: padded length; sc: padded length / group. */
int uq_trellis_normalize(const void *A, int a_dtype, int64_t ntot, int64_t group,
                         int64_t seg, float *xn, float *sc, void *stream);

/* trellis.py:35-42 -- per-row variant used by trellis_quant: rows of T values
 * are padded to Tp = ceil(T / group) * group.  xn: (nrow, Tp), sc:
 * (nrow, Tp / group). */
int uq_trellis_normalize_rows(const void *A, int a_dtype, int64_t nrow, int64_t T,
                              int64_t lda, int64_t group, float *xn, float *sc,
                              void *stream);

/* trellis.py:84-103, qat.py:141-152 -- min-plus Viterbi over `nseq`
 * sequences of T normalised values (xn, row-major).  Writes the full L-bit
 * state of every step: states (nseq, T) int32.  cw: 2^L floats (the
 * codebook, or a tuned one).  6 <= L <= 16, 1 <= R <= 4, L >= 2R, T >= 1.
 * Backpointers live in the caller's workspace (uq_trellis_workspace_bytes). */
size_t uq_trellis_workspace_bytes(int64_t nseq, int T, int L, int R);
int uq_trellis_viterbi(const float *xn, int64_t nseq, int T, int L, int R, const float *cw,
                       int32_t *states, void *workspace, size_t workspace_bytes,
                       void *stream);

/* No counterpart in the reference.  The same Viterbi as uq_trellis_viterbi
 * for callers that cannot allocate device memory (a host that owns all GPU
 * memory through its own allocator and offers plug-ins no allocation hook,
 * or a latency-critical path that must not trigger cudaMalloc's implicit
 * synchronisation).  Backpointers go to a fixed 64 MiB file-scope device
 * array (uq_trellis_noalloc_scratch_bytes()) that each GPU loading the
 * library holds until exit; sequences are processed in batches that fit it.
 * A sequence needing more than that array ((T - 1) * 2^L / 8 bytes at R = 2,
 * 3; half that at R = 1, 4) is rejected
 * with UQ_ERR_INVALID.  Nothing is allocated or freed.  The first call in
 * each CUDA context of a device (the primary context, a new one after
 * cudaDeviceReset, or a caller's own) looks up the array's device address in
 * that context (cudaGetSymbolAddress); make that first call before any
 * stream capture.  Every call shares the array: calls that overlap on the
 * GPU (other streams, other host threads) race.  Throughput: at L = 16,
 * T = 256 one sequence needs ~2 MiB (R = 2, 3), so a batch is 32 sequences,
 * under a quarter of the 148 that one wave of the cluster kernel runs, and
 * each batch ends with a latency-bound traceback launch -- expect about a
 * fifth of the throughput of uq_trellis_viterbi with a workspace there. */
size_t uq_trellis_noalloc_scratch_bytes(void);
int uq_trellis_viterbi_noalloc(const float *xn, int64_t nseq, int T, int L, int R,
                               const float *cw, int32_t *states, void *stream);

/* trellis.py:104-108 -- decoder: out[i] = cw[states[i]] * sc[i / group] for
 * i < ntot (float32 product). */
int uq_trellis_decode(const int32_t *states, const float *cw, const float *sc,
                      int64_t group, int64_t ntot, float *out, void *stream);

/* trellis.py:57-58 -- row decoder of trellis_quant: states (nrow, Tp),
 * sc (nrow, Tp / group); out (nrow, T) = cw[s] * sc cropped to T. */
int uq_trellis_decode_rows(const int32_t *states, const float *cw, const float *sc,
                           int64_t nrow, int64_t T, int64_t Tp, int64_t group,
                           float *out, void *stream);

/* Packed codes of qat.trellis_encode (qat.py:11-33) state paths -- the
 * L + R (T-1) bits per sequence behind the reference's bits-per-weight
 * accounting; no counterpart function in the reference.  A path satisfies
 * s_t = ((s_{t-1} << R) | b_t) mod 2^L, so it is the bit string
 * S = s_0 2^(R(T-1)) + sum_{t>=1} (s_t mod 2^R) 2^(R(T-1-t)), stored least
 * significant 32-bit word first, uq_trellis_packed_words(T, L, R) words per
 * sequence; s_t = (S >> R(T-1-t)) mod 2^L.  Packing keeps only s_0 and the
 * low R bits of later states: states that are not a trellis path (such as
 * the Viterbi kernel's output always is) do not survive a round trip. */
int64_t uq_trellis_packed_words(int T, int L, int R);
int uq_trellis_pack(const int32_t *states, int64_t nseq, int T, int L, int R, uint32_t *packed,
                    void *stream);
int uq_trellis_unpack(const uint32_t *packed, int64_t nseq, int T, int L, int R, int32_t *states,
                      void *stream);

/* ---------------------------------------------------------------------
 * Q8_0 blocks at either side of the path (GGUF container of the builders)
 * ------------------------------------------------------------------- */

/* buildq.py:21-30 enc_q8(W): W (rows, cols) float32 or float64 (converted to
 * float32 first), row stride ldw, cols a multiple of 32; out (rows, cols/32*34)
 * bytes: per block of 32, float16(max|x| / 127, 0 -> 1e-9) little endian,
 * then 32 int8 round-half-even(x / scale) clipped to [-127, 127]. */
int uq_q8_encode(const void *W, int w_dtype, int64_t rows, int64_t cols, int64_t ldw,
                 uint8_t *out, void *stream);

/* qlab.py:27-32 deq_q8(t): blocks as above (rows, cols/32*34 bytes) ->
 * out (rows, cols) float32 = float32(scale) * q, row stride ld_out. */
int uq_q8_decode(const uint8_t *q8, int64_t rows, int64_t cols, float *out, int64_t ld_out,
                 void *stream);

/* ---------------------------------------------------------------------
 * Differentiable decoder of the QAT step (qat.py:35-59)
 * ------------------------------------------------------------------- */

/* qat.py:35-41 fwht_torch / qat.py:43-49 irht_torch, forward (direction 0)
 * and the gradient torch's autograd forms (direction 1).  x: (rows, ncols_in)
 * with row stride ldx, dtype UQ_F32 or UQ_F64 (arithmetic in that dtype),
 * zero-padded to n = 2^k columns (n <= 32768 for f32, <= 16384 for f64).
 * Forward: out = (FWHT(x) / sqrt(n)) [* signs] [/ colscale], first ncols_out
 * columns.  Backward: x is the incoming gradient; out = FWHT^T(((x
 * [/ colscale]) [* signs]) / sqrt(n)) with the stages in reverse order.
 * signs (n) and colscale (ncols) are optional, in the same dtype. */
int uq_fwht(const void *x, int dtype, int64_t rows, int64_t n, int64_t ldx, int64_t ncols_in,
            const void *signs, const void *colscale, int direction, void *out, int64_t ld_out,
            int64_t ncols_out, void *stream);

/* qat.py:51-59 recon_torch: What = irht_torch(cw[states] * sc_g) / sH.
 * states: nrow * n values (int32, or int64 when states64), the flattened
 * rotated matrix (nrow, n); sc: one float per scale_group consecutive
 * values; signs: n floats (+-1); sH: in0 floats (nullable = 1); out (nrow,
 * in0) with row stride ld_out, float32.  A state outside [0, ncw) yields NaN
 * and is reported by uq_device_errors. */
int uq_qat_recon(const void *states, int states64, int64_t nrow, int64_t n, const float *cw,
                 int64_t ncw, const float *sc, int64_t scale_group, const float *signs,
                 const float *sH, int64_t in0, float *out, int64_t ld_out, void *stream);

/* Gradient of recon_torch with respect to cw (ncw floats) and sc_g (ngroups
 * floats) for the incoming gradient grad (nrow, in0), stride ld_grad. */
size_t uq_qat_recon_backward_workspace_bytes(int64_t ncw, int64_t ngroups);
int uq_qat_recon_backward(const float *grad, int64_t ld_grad, const void *states, int states64,
                          int64_t nrow, int64_t n, const float *cw, int64_t ncw,
                          const float *sc, int64_t ngroups, int64_t scale_group,
                          const float *signs, const float *sH, int64_t in0, float *grad_cw,
                          float *grad_sc, void *workspace, size_t workspace_bytes,
                          void *stream);

/* ---------------------------------------------------------------------
 * Importance-weighted pipelines (builder recipes around the path)
 * ------------------------------------------------------------------- */

/* buildtrellis.py:16-20 quant_trellis(W, H): H' = max(H, max(H) * 1e-3),
 * sH = sqrt(H'), A = W * sH, Arot = rht_rows(A), trellis_quant_fast(Arot, L,
 * R, seg, group), Ah = irht_rows(., n0), What = float32(Ah / sH).
 * W: (rows, n0) f32/f64 (stride ldw); H: n0 fp64; signs: n = next_pow2(n0)
 * fp64; cw: 2^L floats.  Outputs: What (rows, n0) float32; optional states
 * (rows * n / seg, seg) int32, sc (rows * n / group) float32 and
 * err[2] fp64 = { sum (A - Ah)^2, sum A^2 } (the weighted NMSE is
 * err[0] / err[1]). */
size_t uq_quant_trellis_workspace_bytes(int64_t rows, int64_t n0, int L, int R, int seg,
                                        int group);
int uq_quant_trellis(const void *W, int w_dtype, int64_t rows, int64_t n0, int64_t ldw,
                     const double *H, int L, int R, int seg, int group,
                     const double *signs, const float *cw, float *What, int32_t *states,
                     float *sc, double *err, void *workspace, size_t workspace_bytes,
                     void *stream);

/* buildalloc.py:21-24 quant_step(W, H, step): same recipe with
 * q_e8_fast(Arot, fixed_step=step, group) in place of the trellis.
 * idx (nullable): 2*pts int16 of the rotated matrix (rows * n values). */
size_t uq_quant_e8_workspace_bytes(int64_t rows, int64_t n0, int group);
int uq_quant_e8(const void *W, int w_dtype, int64_t rows, int64_t n0, int64_t ldw,
                const double *H, double step, int group, const double *signs,
                float *What, int16_t *idx, double *err, void *workspace,
                size_t workspace_bytes, void *stream);

/* qlab.py:53-54 wnmse(A, Ah) = sum((A - Ah)^2) / sum(A^2): out2 = { sum((A -
 * Ah)^2), sum(A^2) } in fp64 over n elements of A and Ah (float32 or fp64,
 * widened exactly); a fixed-order reduction (deterministic for a given n). */
size_t uq_wnmse_workspace_bytes(void);
int uq_wnmse_sums(const void *A, int a_dtype, const void *Ah, int ah_dtype, int64_t n, double *out2,
                  void *workspace, size_t workspace_bytes, void *stream);

/* Opt-in variant of uq_quant_e8 for n0 = 28 x 512 / 28 x 1024 with the
 * block-factorised transform (uq_rht28_rows) in place of the padded RHT and
 * groups of 256; err = { sum (X - Xq)^2, sum X^2 } of the rotated matrix.  No
 * counterpart in the reference. */
size_t uq_quant_e8_b28_workspace_bytes(int64_t rows, int64_t n0);
int uq_quant_e8_b28(const void *W, int w_dtype, int64_t rows, int64_t n0, int64_t ldw,
                    const double *H, double step, const double *signs, float *What, int16_t *idx,
                    double *err, void *workspace, size_t workspace_bytes, void *stream);

/* Opt-in variant of uq_quant_e8 (buildalloc.py:21-24) with the per-row
 * scale search (uq_e8_scale_search) in place of the single step, groups of
 * 256; choice (rows, nullable) and *lam_host as there.  No counterpart in
 * the reference.  Synchronises the stream. */
size_t uq_quant_e8_search_workspace_bytes(int64_t rows, int64_t n0);
int uq_quant_e8_search(const void *W, int w_dtype, int64_t rows, int64_t n0, int64_t ldw,
                       const double *H, double step, const double *signs, float *What, int16_t *idx,
                       int32_t *choice, double *lam_host, double *err, void *workspace,
                       size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------------
 * Device status (no counterpart in the reference)
 * ------------------------------------------------------------------- */

/* Synchronises `stream` and reports (and clears) a timeout of a bounded
 * device wait in the cluster-split Viterbi kernel or the tensor-map RHT / E8
 * kernels (UQ_ERR_TIMEOUT) or a state outside the codebook given to the QAT
 * decoder (UQ_ERR_INVALID) since the last call; else UQ_OK.  A timed-out
 * wait lets its kernel run to the end with wrong results, so callers of
 * uq_quant_trellis / uq_quant_e8 / uq_trellis_viterbi / uq_rht_rows check
 * this before using the outputs (the Python layer does so after every
 * call). */
int uq_device_errors(void *stream);

/* Runs a one-warp kernel that waits on an mbarrier phase nothing completes;
 * the bounded wait gives up after limit_ms (<= 2000).  Returns
 * UQ_ERR_TIMEOUT when the bound worked (the expected outcome). */
int uq_wait_timeout_selftest(double limit_ms, void *stream);

/* Fault injection on the host: sets the timeout flag that a bounded device
 * wait sets when it gives up (which = 0: the cluster-split Viterbi exchange,
 * 1: the tensor-map RHT, 2: the tensor-map E8 quantizer), so that tests can
 * check that the next uq_device_errors reports it.  No kernel runs. */
int uq_inject_device_flag(int which);

/* ---------------------------------------------------------------------
 * Instrumentation (no counterpart in the reference; used by bench.py)
 * ------------------------------------------------------------------- */

/* Count every kernel launch and, when enabled, bracket the launches of the
 * named hot kernels ("viterbi_fwd", "rht", "e8_quant", "traceback") with
 * CUDA events on their launch stream.
 *
 * Independently of this switch, the pipeline entry points, their stages
 * ("rht_forward", "trellis_normalize", "trellis_viterbi", "trellis_decode",
 * "rht_inverse", "e8_quant", "e8_scale_search") and every launch open NVTX
 * ranges in the "ultraquant_b200" domain, for a tracer attached through
 * NVTX_INJECTION64_PATH (no cost beyond a null-pointer check without one). */
void uq_profile_enable(int on);
void uq_profile_reset(void);
int64_t uq_launch_count(void);
/* Synchronises the recorded events of `kernel`; returns the number of
 * launches and their summed device time in milliseconds. */
int uq_profile_read(const char *kernel, double *total_ms, int64_t *launches);

/* Measured denominator of the Viterbi forward's roofline: one launch of a
 * kernel that runs only independent float32 sub / mul / add chains (mode 0:
 * the packed f32x2 forms the Viterbi uses; mode 1: scalar forms) with every
 * SM fully occupied.  Writes the lane operations the launch performs to
 * *lane_ops_host; the caller times the launch with CUDA events on `stream`. */
int uq_fp32_lane_probe(int mode, int64_t iters, double *lane_ops_host, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* UQ_B200_H */
