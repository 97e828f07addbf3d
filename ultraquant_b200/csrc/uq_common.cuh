// Shared helpers of the sm_100a quantization kernels: status/error plumbing,
// exact-rounding arithmetic wrappers and numpy's pairwise summation order.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/uq_b200.h"

namespace uq {

// Records a printf-style message for uq_last_error() and returns `code`.
int fail(int code, const char *fmt, ...);
// Maps the last CUDA error (if any) to UQ_ERR_CUDA with `what` as context.
int check_cuda(const char *what);
// Size in bytes of an element of a uq_dtype, 0 if the code is unknown.
inline int dtype_size(int dt) { return dt == UQ_F32 ? 4 : (dt == UQ_F64 ? 8 : 0); }
inline bool is_pow2(int64_t n) { return n > 0 && (n & (n - 1)) == 0; }
inline int ilog2(int64_t n) { int b = 0; while ((int64_t(1) << b) < n) ++b; return b; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
int num_sms();

// Launch-configuration queries, cached per (kernel, arguments, device, CUDA
// context): the dynamic shared-memory attribute and the occupancy queries are
// host-side driver calls of up to milliseconds each, and every pipeline call
// made several of them.  Without a context ID from the driver they call
// straight through.
cudaError_t set_smem_attr(const void *kernel, int smem);
cudaError_t occupancy_blocks(int *per_sm, const void *kernel, int threads, size_t smem);
cudaError_t occupancy_clusters(int *clusters, const void *kernel, const cudaLaunchConfig_t *cfg);
int qat_take_bad_state();   // uq_qat.cu
int rht_take_timeout();     // uq_rht.cu
int e8_take_timeout();      // uq_e8.cu
int rht_set_timeout();      // uq_rht.cu (fault injection)
int e8_set_timeout();       // uq_e8.cu (fault injection)

// NVTX range in the "ultraquant_b200" domain, open for the object's lifetime
// (host time; a tool such as Nsight Systems attributes the kernels launched
// inside it).  Without an attached tool each push / pop is one call through
// a null function pointer.
struct NvtxRange {
    explicit NvtxRange(const char *name);
    ~NvtxRange();
    NvtxRange(const NvtxRange &) = delete;
    NvtxRange &operator=(const NvtxRange &) = delete;
};

// Launch accounting, an NVTX range named after the kernel, and optional
// per-launch event timing (see uq_profile_*).
void count_launch();
struct ProfScope {
    int slot = -1;
    cudaStream_t st;
    NvtxRange range;
    ProfScope(const char *kernel, cudaStream_t s);  // records a start event if profiling
    ~ProfScope();                                   // records the stop event
};

// Carves aligned sub-buffers out of a caller workspace.
struct Carver {
    char *base;
    size_t cap, off = 0;
    Carver(void *b, size_t c) : base(static_cast<char *>(b)), cap(c) {}
    template <typename T> T *take(size_t count) {
        off = align_up(off, 256);
        T *p = reinterpret_cast<T *>(base ? base + off : nullptr);
        off += count * sizeof(T);
        return p;
    }
    bool ok() const { return off <= cap; }
};

}  // namespace uq

#define UQ_STREAM(s) (static_cast<cudaStream_t>(s))

// ----------------------------------------------------------------------------
// Device helpers
// ----------------------------------------------------------------------------
#if defined(__CUDACC__)

// Explicitly rounded fp ops: never contracted into FMA, so results match a
// sequence of separate numpy / torch element-wise operations.
__device__ __forceinline__ float f_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float f_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float f_mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double d_add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double d_sub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double d_mul(double a, double b) { return __dmul_rn(a, b); }

// numpy's pairwise sum (the order used by add.reduce along a contiguous axis):
//   n < 8:    sequential from 0
//   n <= 128: 8 accumulators r[j] over i = j (mod 8), combined as
//             ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the n % 8 tail
//   n > 128:  split at n2 = n/2 rounded down to a multiple of 8, recurse.
// `get(i)` returns element i.  Used with small n by a single thread.
template <typename T, typename Get>
__device__ T pairwise_leaf(Get get, int64_t off, int64_t n) {
    if (n < 8) {
        T res = T(0);
        for (int64_t i = 0; i < n; ++i) res = res + get(off + i);
        return res;
    }
    T r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = get(off + j);
    int64_t i = 8;
    for (; i < n - (n % 8); i += 8) {
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = r[j] + get(off + i + j);
    }
    T res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res = res + get(off + i);
    return res;
}

// Iterative form of the recursion (explicit stack of pending right halves).
template <typename T, typename Get>
__device__ T pairwise_sum(Get get, int64_t n) {
    // Each frame: (offset, length, partial-left-result, state)
    struct Frame { int64_t off, n; T left; int state; };
    Frame st[24];
    int sp = 0;
    st[0] = {0, n, T(0), 0};
    T ret = T(0);
    while (sp >= 0) {
        Frame &f = st[sp];
        if (f.n <= 128) {
            ret = pairwise_leaf<T>(get, f.off, f.n);
            --sp;
            // deliver ret to parent
            while (sp >= 0) {
                Frame &p = st[sp];
                if (p.state == 1) {  // left done, now run right
                    p.left = ret;
                    p.state = 2;
                    int64_t n2 = p.n / 2;
                    n2 -= n2 % 8;
                    st[++sp] = {p.off + n2, p.n - n2, T(0), 0};
                    break;
                } else {             // right done
                    ret = p.left + ret;
                    --sp;
                }
            }
        } else {
            int64_t n2 = f.n / 2;
            n2 -= n2 % 8;
            f.state = 1;
            st[++sp] = {f.off, n2, T(0), 0};
        }
    }
    return ret;
}
#endif  // __CUDACC__
