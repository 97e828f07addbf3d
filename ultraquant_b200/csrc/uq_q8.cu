// Q8_0 blocks around the quantization path for sm_100a:
//
//   enc_q8  buildq.py:21-30  x = float32(W) in blocks of 32 along a row,
//                            sc = max|x| / 127 (sc == 0 -> 1e-9),
//                            q = round-half-even(x / sc) clipped to [-127, 127],
//                            block = float16(sc) (2 bytes, little endian) + 32 int8
//   deq_q8  qlab.py:27-32    W = float32(float16 scale) * float32(q)
//
// Every step is one correctly rounded float32 (or float16 conversion)
// operation, so the bytes and values are the reference's.  One warp per
// 32-block span of a row: lane l holds element l of each block (coalesced
// loads), the block maximum is a shuffle reduction (max is exact), the 32
// quantized bytes of a block are one coalesced 32-byte store.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <stdint.h>

#include "uq_common.cuh"

namespace {

constexpr int kBlk = 32, kBlkBytes = 34, kSpan = 32;   // blocks per warp task

template <typename T>
__global__ void q8_encode_kernel(const T *W, int64_t rows, int64_t nb, int64_t ld, uint8_t *out) {
    const int lane = threadIdx.x & 31;
    const int64_t spans = (nb + kSpan - 1) / kSpan;
    const int64_t tasks = rows * spans;
    const int64_t warp0 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t task = warp0; task < tasks; task += nwarps) {
        const int64_t r = task / spans, b0 = (task % spans) * kSpan;
        const int nblk = int(std::min<int64_t>(kSpan, nb - b0));
        const T *src = W + r * ld + b0 * kBlk;
        uint8_t *dst = out + (r * nb + b0) * kBlkBytes;
        float x[kSpan];
#pragma unroll
        for (int j = 0; j < kSpan; ++j) x[j] = j < nblk ? float(__ldg(src + j * kBlk + lane)) : 0.f;
#pragma unroll
        for (int j = 0; j < kSpan; ++j) {
            if (j >= nblk) break;
            float m = fabsf(x[j]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            float sc = __fdiv_rn(m, 127.0f);
            if (sc == 0.0f) sc = 1e-9f;
            float q = rintf(__fdiv_rn(x[j], sc));
            q = fminf(fmaxf(q, -127.0f), 127.0f);
            dst[j * kBlkBytes + 2 + lane] = uint8_t(int8_t(int(q)));
            if (lane == 0) {
                // float16 scale, little endian; blocks start on even bytes
                *reinterpret_cast<unsigned short *>(dst + j * kBlkBytes) = __half_as_ushort(__float2half_rn(sc));
            }
        }
    }
}

__global__ void q8_decode_kernel(const uint8_t *q8, int64_t rows, int64_t nb, float *out, int64_t ld_out) {
    const int64_t total = rows * nb * kBlk;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t blk = i / kBlk;                 // row-major block index
        const int e = int(i % kBlk);
        const uint8_t *bp = q8 + blk * kBlkBytes;
        const unsigned short h = static_cast<unsigned short>(__ldg(bp) | (__ldg(bp + 1) << 8));
        const float sc = __half2float(__ushort_as_half(h));
        const float q = float(int8_t(__ldg(bp + 2 + e)));
        const int64_t r = blk / nb, c = (blk % nb) * kBlk + e;
        out[r * ld_out + c] = __fmul_rn(sc, q);
    }
}

int grid_for(int64_t work, int per_block) {
    return int(std::max<int64_t>(1, std::min<int64_t>((work + per_block - 1) / per_block, int64_t(uq::num_sms()) * 16)));
}

}  // namespace

extern "C" {

int uq_q8_encode(const void *W, int w_dtype, int64_t rows, int64_t cols, int64_t ldw, uint8_t *out, void *stream) {
    if (rows < 0 || cols < 0 || cols % kBlk || ldw < cols || !uq::dtype_size(w_dtype))
        return uq::fail(UQ_ERR_INVALID, "uq_q8_encode: bad shape (rows=%lld cols=%lld ld=%lld; cols must be a multiple of 32)",
                        (long long)rows, (long long)cols, (long long)ldw);
    if (rows == 0 || cols == 0) return UQ_OK;
    if (!W || !out) return uq::fail(UQ_ERR_INVALID, "uq_q8_encode: null pointer");
    const int64_t nb = cols / kBlk;
    const int64_t tasks = rows * ((nb + kSpan - 1) / kSpan);
    const int grid = grid_for(tasks, 8);
    const cudaStream_t st = UQ_STREAM(stream);
    {
        uq::ProfScope _p("q8_encode", st);
        if (w_dtype == UQ_F32) q8_encode_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float *>(W), rows, nb, ldw, out);
        else q8_encode_kernel<double><<<grid, 256, 0, st>>>(static_cast<const double *>(W), rows, nb, ldw, out);
    }
    return uq::check_cuda("q8_encode_kernel launch");
}

int uq_q8_decode(const uint8_t *q8, int64_t rows, int64_t cols, float *out, int64_t ld_out, void *stream) {
    if (rows < 0 || cols < 0 || cols % kBlk || ld_out < cols)
        return uq::fail(UQ_ERR_INVALID, "uq_q8_decode: bad shape (rows=%lld cols=%lld ld=%lld; cols must be a multiple of 32)",
                        (long long)rows, (long long)cols, (long long)ld_out);
    if (rows == 0 || cols == 0) return UQ_OK;
    if (!q8 || !out) return uq::fail(UQ_ERR_INVALID, "uq_q8_decode: null pointer");
    const int grid = grid_for(rows * cols, 256);
    { uq::ProfScope _p("q8_decode", UQ_STREAM(stream)); q8_decode_kernel<<<grid, 256, 0, UQ_STREAM(stream)>>>(q8, rows, cols / kBlk, out, ld_out); }
    return uq::check_cuda("q8_decode_kernel launch");
}

}  // extern "C"
