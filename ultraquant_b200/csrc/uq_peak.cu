// FP32 lane-throughput probe: the measured denominator of the Viterbi
// forward's roofline.
//
// The Viterbi forward spends its algorithmic work on packed float32
// sub / mul / add (sub.rn.f32x2, mul.rn.f32x2, add.rn.f32x2; never fused), so
// the probe runs exactly that instruction mix: every thread carries eight
// independent chains a <- (a - c) * h + c, each link one packed sub, one packed
// multiply (an FMA with a +0 addend, as the Viterbi forms its squares) and one
// packed add (6 lane operations), with enough resident warps
// and independent chains that no dependency latency is exposed.  The caller
// times one launch with CUDA events on `stream`; lane operations / time is the
// achievable FP32 lane rate of this GPU at its current clocks.  Mode 1 runs
// the same chains with scalar (unpacked) float32 instructions.
#include <cuda_runtime.h>

#include "uq_common.cuh"

namespace {

typedef unsigned long long u64;

__device__ float g_peak_sink;

__device__ __forceinline__ u64 p_pk2(float lo, float hi) {
    u64 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ u64 p_sub2(u64 a, u64 b) {
    u64 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// RN(a * b) as a packed FMA with a +0 addend, the Viterbi's form of its
// squares: ptxas fuses a mul.rn.f32x2 feeding an add.rn.f32x2 into one FMA
// (even with -fmad=false), which would make each link two instructions and
// overstate the rate of three separately rounded operations by 1.5x.
__device__ __forceinline__ u64 p_mul2(u64 a, u64 b) {
    u64 r;
    const u64 zero = 0ull;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(zero));
    return r;
}
__device__ __forceinline__ u64 p_add2(u64 a, u64 b) {
    u64 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

constexpr int kChains = 8;
constexpr int kThreadsPerBlock = 256;
constexpr int kUnroll = 4;

__global__ void __launch_bounds__(kThreadsPerBlock) fp32_lane_probe_packed(int iters, float c0) {
    u64 a[kChains];
    const float base = float(threadIdx.x) * 1e-7f;
#pragma unroll
    for (int i = 0; i < kChains; ++i) a[i] = p_pk2(base + float(i) * 1e-3f, base - float(i) * 1e-3f);
    const u64 c = p_pk2(c0, -c0), h = p_pk2(0.5f, 0.5f);
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
#pragma unroll
            for (int i = 0; i < kChains; ++i) a[i] = p_add2(p_mul2(p_sub2(a[i], c), h), c);
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kChains; ++i) {
        float lo, hi;
        asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(a[i]));
        s += lo + hi;
    }
    if (s == 1234.5f) g_peak_sink = s;   // keeps the chains live; never true for these inputs
}

__global__ void __launch_bounds__(kThreadsPerBlock) fp32_lane_probe_scalar(int iters, float c0) {
    float a[2 * kChains];
    const float base = float(threadIdx.x) * 1e-7f;
#pragma unroll
    for (int i = 0; i < 2 * kChains; ++i) a[i] = base + float(i) * 1e-3f;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
#pragma unroll
            for (int i = 0; i < 2 * kChains; ++i) a[i] = __fadd_rn(__fmul_rn(__fsub_rn(a[i], c0), 0.5f), c0);
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 2 * kChains; ++i) s += a[i];
    if (s == 1234.5f) g_peak_sink = s;
}

}  // namespace

extern "C" int uq_fp32_lane_probe(int mode, int64_t iters, double *lane_ops_host, void *stream) {
    if ((mode != 0 && mode != 1) || iters < 1 || iters > (int64_t(1) << 30) || !lane_ops_host)
        return uq::fail(UQ_ERR_INVALID, "uq_fp32_lane_probe: bad arguments (mode=%d iters=%lld)", mode,
                        (long long)iters);
    cudaStream_t st = UQ_STREAM(stream);
    // eight 256-thread CTAs per SM: 2,048 resident threads, the SM's maximum
    const int blocks = uq::num_sms() * 8;
    {
        uq::ProfScope _p("fp32_probe", st);
        if (mode == 0) fp32_lane_probe_packed<<<blocks, kThreadsPerBlock, 0, st>>>(int(iters), 0.75f);
        else fp32_lane_probe_scalar<<<blocks, kThreadsPerBlock, 0, st>>>(int(iters), 0.75f);
    }
    // 16 lanes per thread (8 packed chains of 2), 3 operations per link
    *lane_ops_host = double(blocks) * kThreadsPerBlock * double(iters) * kUnroll * (2 * kChains) * 3.0;
    return uq::check_cuda("fp32_lane_probe launch");
}
