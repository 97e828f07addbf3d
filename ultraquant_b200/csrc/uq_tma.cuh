// Tensor-memory-accelerator (TMA) and mbarrier helpers shared by the
// transform and quantizer kernels: bounded mbarrier waits, tensor-map
// loads / stores into the issuing CTA's own shared memory, bulk-group bookkeeping and
// the host-side tensor-map encoder (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the library needs no libcuda link).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <stdint.h>

namespace uq {
namespace tma {

#if defined(__CUDACC__)
__device__ __forceinline__ void mbar_init(unsigned addr, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(addr), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned addr, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(addr), "r"(bytes) : "memory");
}
// Waits for the phase with the given parity, at most ~2 s; then records the
// timeout in *flag, sets `fail` (later waits return at once) and returns.
__device__ __forceinline__ void mbar_wait_bounded(unsigned addr, unsigned parity, bool &fail, int *flag) {
    if (fail) return;
    unsigned long long t0 = 0;
    for (unsigned it = 0;; ++it) {
        unsigned done;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(done) : "r"(addr), "r"(parity) : "memory");
        if (done) return;
        if ((it & 63) == 0) {
            unsigned long long now;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
            if (it == 0) t0 = now;
            else if (now - t0 > 2000000000ull) {
                fail = true;
                atomicExch(flag, 1);
                return;
            }
        }
    }
}
__device__ __forceinline__ void load2d(unsigned dst, const CUtensorMap *map, int c0, int c1, unsigned mbar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 :: "r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(mbar) : "memory");
}
__device__ __forceinline__ void store2d(const CUtensorMap *map, int c0, int c1, unsigned src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                 :: "l"(map), "r"(c0), "r"(c1), "r"(src) : "memory");
}
__device__ __forceinline__ void load3d(unsigned dst, const CUtensorMap *map, int c0, int c1, int c2, unsigned mbar) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
                 :: "r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(mbar) : "memory");
}
__device__ __forceinline__ void store3d(const CUtensorMap *map, int c0, int c1, int c2, unsigned src) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                 :: "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(src) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ float4 lds128f(unsigned addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ double2 lds128d(unsigned addr) {
    double2 v;
    asm volatile("ld.shared.v2.f64 {%0,%1}, [%2];" : "=d"(v.x), "=d"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ double lds64d(unsigned addr) {
    double v;
    asm volatile("ld.shared.f64 %0, [%1];" : "=d"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ void sts128d(unsigned addr, double a, double b) {
    asm volatile("st.shared.v2.f64 [%0], {%1, %2};" :: "r"(addr), "d"(a), "d"(b) : "memory");
}
// Byte offset of element e of a buffer of 128-byte lines written with the
// 128-byte swizzle (16-byte chunk c of line r stored at chunk c ^ (r & 7)).
template <typename T> __device__ __forceinline__ unsigned swz128(int e) {
    constexpr int EPL = 128 / int(sizeof(T));
    constexpr int EPC = 16 / int(sizeof(T));
    const int r = e / EPL, c = (e % EPL) / EPC;
    return unsigned(r * 128 + ((c ^ (r & 7)) << 4) + (e % EPC) * int(sizeof(T)));
}
#endif  // __CUDACC__

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// Tiled map with the 128-byte swizzle and zero fill; dims[0] * element size
// must be 128 bytes (one line).  strides: rank - 1 byte strides of dims 1...
inline bool encode_lines(CUtensorMap *m, bool f64, int rank, const void *base, const cuuint64_t *dims,
                         const cuuint64_t *strides, const cuuint32_t *box) {
    EncodeTiled fn = encode_fn();
    if (!fn) return false;
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return fn(m, f64 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT64 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, cuuint32_t(rank),
              const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tma
}  // namespace uq
