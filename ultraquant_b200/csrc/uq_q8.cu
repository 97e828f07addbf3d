// Q8_0 blocks around the quantization path for sm_100a:
//
//   enc_q8  buildq.py:21-30  x = float32(W) in blocks of 32 along a row,
//                            sc = max|x| / 127 (sc == 0 -> 1e-9),
//                            q = round-half-even(x / sc) clipped to [-127, 127],
//                            block = float16(sc) (2 bytes, little endian) + 32 int8
//   deq_q8  qlab.py:27-32    W = float32(float16 scale) * float32(q)
//
// Every step is one correctly rounded float32 (or float16 conversion)
// operation, so the bytes and values are the reference's.  Both kernels move
// spans of 256 blocks (8704 bytes, a multiple of 16) through shared memory so
// that the byte-granular block format meets global memory as 16-byte
// vectors; the block maximum is a shuffle reduction over the 4 threads of a
// block (max is exact).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <stdint.h>

#include "uq_common.cuh"

namespace {

constexpr int kBlk = 32, kBlkBytes = 34;
constexpr int kSpan = 256;                          // blocks per CTA task
constexpr int kSpanBytes = kSpan * kBlkBytes;       // 8704 = 544 x 16 bytes

// Element i (< 32) of block gb of a (rows, nb * 32) matrix with row stride ld.
__device__ __forceinline__ int64_t blk_base(int64_t gb, int64_t nb, int64_t ld) {
    return (gb / nb) * ld + (gb % nb) * kBlk;
}

// 256 threads, 4 per block: lane group (tid >> 2) quantizes one block per pass,
// each thread 8 elements (two 16-byte loads), so a block's scale and
// reciprocal are computed once per 8 values; the span's 34-byte blocks are
// staged in shared memory and leave as 16-byte stores.
constexpr int kTPB = 4, kVPT = kBlk / kTPB, kPasses = kSpan / (256 / kTPB);

template <typename T>
__global__ void __launch_bounds__(256) q8_encode_kernel(const T *W, int64_t nblocks, int64_t nb, int64_t ld,
                                                        bool vec_in, uint8_t *out, bool vec_out) {
    __shared__ __align__(16) uint8_t stage[kSpanBytes];
    const int tid = threadIdx.x, sub = tid & (kTPB - 1);
    for (int64_t b0 = int64_t(blockIdx.x) * kSpan; b0 < nblocks; b0 += int64_t(gridDim.x) * kSpan) {
        const int nblk = int(nblocks - b0 < kSpan ? nblocks - b0 : int64_t(kSpan));
        // all of the thread's loads of the span first (4 passes x 8 values)
        float xs[kPasses][kVPT];
#pragma unroll
        for (int pass = 0; pass < kPasses; ++pass) {
            const int j = pass * (256 / kTPB) + tid / kTPB;
#pragma unroll
            for (int i = 0; i < kVPT; ++i) xs[pass][i] = 0.f;
            if (j < nblk) {
                const T *src = W + blk_base(b0 + j, nb, ld) + kVPT * sub;
                if (sizeof(T) == 4 && vec_in) {
#pragma unroll
                    for (int h = 0; h < kVPT / 4; ++h) {
                        const float4 v = __ldg(reinterpret_cast<const float4 *>(src) + h);
                        xs[pass][4 * h] = v.x; xs[pass][4 * h + 1] = v.y; xs[pass][4 * h + 2] = v.z; xs[pass][4 * h + 3] = v.w;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < kVPT; ++i) xs[pass][i] = float(__ldg(src + i));
                }
            }
        }
#pragma unroll
        for (int pass = 0; pass < kPasses; ++pass) {
            const int j = pass * (256 / kTPB) + tid / kTPB;
            const bool ok = j < nblk;
            const float *x = xs[pass];
            float m = fabsf(x[0]);
#pragma unroll
            for (int i = 1; i < kVPT; ++i) m = fmaxf(m, fabsf(x[i]));
#pragma unroll
            for (int o = kTPB / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            // sc = RN(m / 127): Markstein's correction (P. Markstein, IBM J. Res.
            // Dev. 34(1), 1990) of q0 = RN(m y), y = RN(1/127): the remainder
            // m - q0 127 is exact as an FMA and RN(q0 + r y) is the correctly
            // rounded quotient while nothing leaves the normal range; other m
            // take the IEEE division
            constexpr float y127 = 1.0f / 127.0f;
            const float q0 = __fmul_rn(m, y127);
            float sc = __fmaf_rn(__fmaf_rn(-q0, 127.0f, m), y127, q0);
            if (!(m >= 0x1p-100f && m <= 0x1p100f)) sc = __fdiv_rn(m, 127.0f);
            if (sc == 0.0f) sc = 1e-9f;
            // rint(x / sc) from t = x * rc, rc the hardware reciprocal (rcp.approx,
            // within 1 ulp of 1/sc): |t - x/sc| <= |x/sc| (2^-23 + 2^-24) (1 + 2^-23)
            // < 2^-15 for |x/sc| <= 127 (1 + 2^-23), so rint(t) is the answer
            // unless t lies within 2^-15 of a rounding boundary (then: the IEEE
            // division).  A subnormal sc flushes to an infinite rc: no t passes.
            float rc;
            asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(rc) : "f"(sc));
            if (ok) {
                // rint(t) as (t + 1.5 2^23) - 1.5 2^23: for |t| < 2^22 the sum lies
                // in [2^23, 2^24), where the spacing is 1, so round-to-nearest-even
                // of the addition is rint(t), and the sum's low byte is rint(t)
                // as a two's-complement int8 (1.5 2^23 = 0x4B400000 ends in 0x00)
                constexpr float kMagic = 12582912.0f;
                int qq[kVPT];
                bool bad = false;
#pragma unroll
                for (int e = 0; e < kVPT; ++e) {
                    const float t = __fmul_rn(x[e], rc);
                    const float sm = __fadd_rn(t, kMagic);
                    const float f = __fsub_rn(sm, kMagic);
                    // (NaN / inf t, from a huge reciprocal, also fail the test)
                    bad |= !(__fsub_rn(0.5f, fabsf(__fsub_rn(t, f))) > 0x1p-15f);
                    qq[e] = int(__float_as_uint(sm));
                }
                if (bad) {
                    // |x / sc| <= 127 (1 + 2^-23): the quotient rounds into [-127, 127]
#pragma unroll
                    for (int e = 0; e < kVPT; ++e) qq[e] = __float2int_rn(rintf(__fdiv_rn(x[e], sc)));
                }
                // block j starts on an even byte: 16-bit stores
                unsigned short *bq = reinterpret_cast<unsigned short *>(stage + j * kBlkBytes + 2 + kVPT * sub);
#pragma unroll
                for (int h = 0; h < kVPT / 2; ++h) bq[h] = static_cast<unsigned short>(__byte_perm(qq[2 * h], qq[2 * h + 1], 0x0040));
                if (sub == 0) *reinterpret_cast<unsigned short *>(stage + j * kBlkBytes) = __half_as_ushort(__float2half_rn(sc));
            }
        }
        __syncthreads();
        const int nbytes = nblk * kBlkBytes;
        uint8_t *dst = out + b0 * kBlkBytes;
        if (vec_out) {
            for (int v = tid; v < nbytes / 16; v += blockDim.x)
                reinterpret_cast<uint4 *>(dst)[v] = reinterpret_cast<const uint4 *>(stage)[v];
            for (int i = (nbytes / 16) * 16 + tid; i < nbytes; i += blockDim.x) dst[i] = stage[i];
        } else {
            for (int i = tid; i < nbytes; i += blockDim.x) dst[i] = stage[i];
        }
        __syncthreads();
    }
}

// The span's bytes come in by 16-byte loads into shared memory; each thread
// then emits float4s of one block (fp32 product of the float16 scale and q).
__global__ void __launch_bounds__(256) q8_decode_kernel(const uint8_t *q8, int64_t nblocks, int64_t nb, bool vec_in,
                                                        float *out, int64_t ld_out, bool vec_out) {
    __shared__ __align__(16) uint8_t stage[kSpanBytes];
    const int tid = threadIdx.x;
    for (int64_t b0 = int64_t(blockIdx.x) * kSpan; b0 < nblocks; b0 += int64_t(gridDim.x) * kSpan) {
        const int nblk = int(nblocks - b0 < kSpan ? nblocks - b0 : int64_t(kSpan));
        const int nbytes = nblk * kBlkBytes;
        const uint8_t *src = q8 + b0 * kBlkBytes;
        if (vec_in) {
            for (int v = tid; v < nbytes / 16; v += blockDim.x)
                reinterpret_cast<uint4 *>(stage)[v] = __ldg(reinterpret_cast<const uint4 *>(src) + v);
            for (int i = (nbytes / 16) * 16 + tid; i < nbytes; i += blockDim.x) stage[i] = __ldg(src + i);
        } else {
            for (int i = tid; i < nbytes; i += blockDim.x) stage[i] = __ldg(src + i);
        }
        __syncthreads();
        for (int f = tid; f < nblk * 8; f += blockDim.x) {
            const int j = f >> 3, sub = f & 7;
            const uint8_t *bp = stage + j * kBlkBytes;
            const float sc = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(bp)));
            const unsigned short *bq = reinterpret_cast<const unsigned short *>(bp + 2 + 4 * sub);
            const unsigned short q01 = bq[0], q23 = bq[1];
            const float4 o = make_float4(__fmul_rn(sc, float(int8_t(q01 & 0xff))), __fmul_rn(sc, float(int8_t(q01 >> 8))),
                                         __fmul_rn(sc, float(int8_t(q23 & 0xff))), __fmul_rn(sc, float(int8_t(q23 >> 8))));
            float *dst = out + blk_base(b0 + j, nb, ld_out) + 4 * sub;
            if (vec_out) {
                *reinterpret_cast<float4 *>(dst) = o;
            } else {
                dst[0] = o.x; dst[1] = o.y; dst[2] = o.z; dst[3] = o.w;
            }
        }
        __syncthreads();
    }
}

// One wave of resident CTAs (persistent grid-stride over spans): a second,
// partial wave would leave SMs idle at the end.
template <typename K>
int grid_for(K kern, int64_t work, int per_block) {
    int per_sm = 0;
    if (uq::occupancy_blocks(&per_sm, reinterpret_cast<const void *>(kern), 256, 0) != cudaSuccess || per_sm < 1) per_sm = 1;
    return int(std::max<int64_t>(1, std::min<int64_t>((work + per_block - 1) / per_block,
                                                      int64_t(uq::num_sms()) * per_sm)));
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

int uq_q8_encode(const void *W, int w_dtype, int64_t rows, int64_t cols, int64_t ldw, uint8_t *out, void *stream) {
    if (rows < 0 || cols < 0 || cols % kBlk || ldw < cols || !uq::dtype_size(w_dtype))
        return uq::fail(UQ_ERR_INVALID, "uq_q8_encode: bad shape (rows=%lld cols=%lld ld=%lld; cols must be a multiple of 32)",
                        (long long)rows, (long long)cols, (long long)ldw);
    if (rows == 0 || cols == 0) return UQ_OK;
    if (!W || !out) return uq::fail(UQ_ERR_INVALID, "uq_q8_encode: null pointer");
    const int64_t nb = cols / kBlk, nblocks = rows * nb;
    const cudaStream_t st = UQ_STREAM(stream);
    const bool vec_out = al16(out);
    {
        uq::ProfScope _p("q8_encode", st);
        if (w_dtype == UQ_F32) {
            const bool vec_in = al16(W) && ldw % 4 == 0;
            const int grid = grid_for(q8_encode_kernel<float>, nblocks, kSpan);
            q8_encode_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float *>(W), nblocks, nb, ldw, vec_in, out, vec_out);
        } else {
            const int grid = grid_for(q8_encode_kernel<double>, nblocks, kSpan);
            q8_encode_kernel<double><<<grid, 256, 0, st>>>(static_cast<const double *>(W), nblocks, nb, ldw, false, out, vec_out);
        }
    }
    return uq::check_cuda("q8_encode_kernel launch");
}

int uq_q8_decode(const uint8_t *q8, int64_t rows, int64_t cols, float *out, int64_t ld_out, void *stream) {
    if (rows < 0 || cols < 0 || cols % kBlk || ld_out < cols)
        return uq::fail(UQ_ERR_INVALID, "uq_q8_decode: bad shape (rows=%lld cols=%lld ld=%lld; cols must be a multiple of 32)",
                        (long long)rows, (long long)cols, (long long)ld_out);
    if (rows == 0 || cols == 0) return UQ_OK;
    if (!q8 || !out) return uq::fail(UQ_ERR_INVALID, "uq_q8_decode: null pointer");
    const int64_t nb = cols / kBlk, nblocks = rows * nb;
    const int grid = grid_for(q8_decode_kernel, nblocks, kSpan);
    const bool vec_out = al16(out) && ld_out % 4 == 0;
    { uq::ProfScope _p("q8_decode", UQ_STREAM(stream)); q8_decode_kernel<<<grid, 256, 0, UQ_STREAM(stream)>>>(q8, nblocks, nb, al16(q8), out, ld_out, vec_out); }
    return uq::check_cuda("q8_decode_kernel launch");
}

}  // extern "C"
