// Per-group sum of squares in numpy's pairwise order, computed cooperatively
// by a CTA on a tile held in shared memory.
//
// For a power-of-two group G the numpy recursion splits into leaves of
// min(G, 128) elements combined by a balanced binary tree; a leaf is 8
// sequential accumulator chains (element j, j+8, j+16, ...) combined as
// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) -- exactly a xor-1/2/4 shuffle tree
// over 8 lanes (IEEE addition is commutative).  Other group sizes (multiples
// of 8) fall back to one thread per group running the generic recursion.
#pragma once
#include "uq_common.cuh"

template <typename T>
__device__ __forceinline__ T sq_rn(T v);
template <> __device__ __forceinline__ float sq_rn<float>(float v) { return __fmul_rn(v, v); }
template <> __device__ __forceinline__ double sq_rn<double>(double v) { return __dmul_rn(v, v); }

// tile: shared memory, `ngroups * group` elements.  out: ngroups sums in
// shared memory.  scratch: shared memory of at least ngroups * 32 elements.
// Must be called by all threads of the CTA; ends with __syncthreads().
template <typename T>
__device__ void tile_group_sumsq(const T *tile, int ngroups, int group, T *out, T *scratch) {
    const int tid = threadIdx.x, nthr = blockDim.x;
    const bool pow2 = (group & (group - 1)) == 0;
    if (pow2 && group >= 8 && group <= 4096) {
        const int leaf = group < 128 ? group : 128;
        const int nleaf = group / leaf;                 // <= 32
        const int lanes_per_group = 8 * nleaf;          // <= 256
        const int total = ngroups * lanes_per_group;    // multiple of 8
        const int iters = leaf / 8;
        for (int base = 0; base < total; base += nthr) {
            // all lanes of a warp stay active so the shuffles are well defined
            const int w = base + tid;
            const bool act = w < total;
            const int g = act ? w / lanes_per_group : 0;
            const int rem = w - g * lanes_per_group;
            const int lf = rem >> 3, j = rem & 7;
            T r = T(0);
            if (act) {
                const T *p = tile + size_t(g) * group + lf * leaf + j;
                r = sq_rn<T>(p[0]);
                for (int i = 1; i < iters; ++i) r = r + sq_rn<T>(p[8 * i]);
            }
            r = r + __shfl_xor_sync(0xffffffffu, r, 1);
            r = r + __shfl_xor_sync(0xffffffffu, r, 2);
            r = r + __shfl_xor_sync(0xffffffffu, r, 4);
            if (act && j == 0) scratch[g * 32 + lf] = r;
        }
        __syncthreads();
        for (int g = tid; g < ngroups; g += nthr) {
            T *s = scratch + g * 32;
            for (int width = nleaf; width > 1; width >>= 1)
                for (int i = 0; i < width / 2; ++i) s[i] = s[2 * i] + s[2 * i + 1];
            out[g] = s[0];
        }
    } else {
        for (int g = tid; g < ngroups; g += nthr) {
            const T *p = tile + size_t(g) * group;
            out[g] = pairwise_sum<T>([p](int64_t i) { return sq_rn<T>(p[i]); }, group);
        }
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// Warp-level form for power-of-two groups G in [8, 256].
//
// Phase 1 ("chain layout"): a group occupies LPG = 8 * NLEAF lanes, lane
// (leaf lf, chain j) loads the leaf's elements j, j+8, j+16, ... and adds their
// squares sequentially (numpy's 8 accumulators), then xor-shuffles 1, 2, 4
// combine the 8 chains as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) and xor 8 adds
// the two 128-leaves.  Every lane of the group ends with the group sum.
// ---------------------------------------------------------------------------
template <int G> struct WarpGroup {
    static_assert(G >= 8 && G <= 256 && (G & (G - 1)) == 0, "power-of-two group in [8, 256]");
    static constexpr int LEAF = G < 128 ? G : 128;
    static constexpr int NLEAF = G / LEAF;       // 1 or 2
    static constexpr int LPG = 8 * NLEAF;        // lanes per group in the chain layout
    static constexpr int GPW = 32 / LPG;         // groups per warp
    static constexpr int CH = LEAF / 8;          // chain length
    static constexpr int VPG = G / 8;            // 8-vectors per group
    static constexpr int VPW = GPW * VPG;        // 8-vectors per warp
};

// Sum of squares of group (g0 + lane / LPG), elements read by get(i) with
// i relative to the warp's first element (g0 * G); identical in all lanes of
// the group.  Must be called by the full warp.
template <int G, typename T, typename Get>
__device__ __forceinline__ T warp_group_sumsq(Get get) {
    using W = WarpGroup<G>;
    const int lane = threadIdx.x & 31;
    const int gl = lane / W::LPG, lf = (lane % W::LPG) / 8, j = lane & 7;
    const int base = gl * G + lf * W::LEAF + j;
    T v0 = get(base);
    T r = sq_rn<T>(v0);
#pragma unroll
    for (int i = 1; i < W::CH; ++i) r = r + sq_rn<T>(get(base + 8 * i));
    r = r + __shfl_xor_sync(0xffffffffu, r, 1);
    r = r + __shfl_xor_sync(0xffffffffu, r, 2);
    r = r + __shfl_xor_sync(0xffffffffu, r, 4);
    if (W::NLEAF == 2) r = r + __shfl_xor_sync(0xffffffffu, r, 8);
    return r;
}
