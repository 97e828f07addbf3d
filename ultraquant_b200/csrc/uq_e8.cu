// E8 nearest-point quantizer (qlab.py:133-183) for sm_100a.
//
// q_e8_fast: per-group RMS in fp64 (numpy pairwise order), gn = g / rms,
// Y = gn / step, closed-form Conway-Sloane decode of D8 u (D8 + 1/2), then
// rec = (pts * step) * rms.  All fp64 operations are the reference's, one by
// one, with IEEE division and no FMA contraction, so points and
// reconstructions are bit-exact.  The kernel is HBM-bound: a CTA stages a
// tile of whole groups in shared memory (coalesced), reduces the group RMS
// cooperatively, then every thread decodes one 8-vector.
//
// Entropy (qlab.py:151-156): distinct 8-tuples of 2*pts are counted in an
// open-addressing hash table (64-bit keys, one byte per coordinate), the
// rate -sum p log2 p is accumulated in 2^-64 fixed point (order independent,
// hence deterministic) and divided by 8.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "uq_common.cuh"
#include "uq_e8core.cuh"
#include "uq_groupsum.cuh"
#include "uq_tma.cuh"
#include "uq_mt19937.h"

namespace {

__global__ void d8_kernel(const double *Y, int64_t nvec, double *out, int e8) {
    for (int64_t v = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; v < nvec;
         v += int64_t(gridDim.x) * blockDim.x) {
        double y[8], p[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = __ldg(Y + 8 * v + i);
        if (e8) e8_point(y, p); else d8_point(y, p);
#pragma unroll
        for (int i = 0; i < 8; ++i) out[8 * v + i] = p[i];
    }
}

// ---- fixed-step quantizer ---------------------------------------------------
struct E8Args {
    const void *A;
    int64_t size;      // valid elements
    int group;
    int tile;          // elements per CTA (multiple of group and of 8)
    double step;
    double *rec;       // size
    int16_t *idx;      // padded size, nullable
    double *rms_out;   // per group, nullable (calibration uses it)
};

template <typename TIn>
__global__ void e8_quant_kernel(E8Args a) {
    extern __shared__ double sm[];
    double *tile = sm;                       // a.tile
    const int ng = a.tile / a.group;
    double *rms = tile + a.tile;             // ng
    double *scratch = rms + ng;              // ng * 32
    const int64_t base = int64_t(blockIdx.x) * a.tile;
    const TIn *A = static_cast<const TIn *>(a.A);
    for (int i = threadIdx.x; i < a.tile; i += blockDim.x) {
        const int64_t gi = base + i;
        tile[i] = gi < a.size ? double(__ldg(A + gi)) : 0.0;
    }
    __syncthreads();
    tile_group_sumsq<double>(tile, ng, a.group, rms, scratch);
    for (int g = threadIdx.x; g < ng; g += blockDim.x) {
        // np.sqrt((g**2).mean()) + 1e-12: mean = sum / count in fp64
        const double r = d_add(sqrt(rms[g] / double(a.group)), 1e-12);
        rms[g] = r;
        if (a.rms_out) {
            const int64_t gg = base / a.group + g;
            if (gg * a.group < a.size) a.rms_out[gg] = r;
        }
    }
    __syncthreads();
    if (!a.rec && !a.idx) return;
    for (int v = threadIdx.x; v < a.tile / 8; v += blockDim.x) {
        const int64_t e0 = base + 8 * int64_t(v);
        if (e0 >= a.size) break;
        const double r = rms[(8 * v) / a.group];
        double y[8], p[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = (tile[8 * v + i] / r) / a.step;
        e8_point(y, p);
        if (a.rec) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (e0 + i < a.size) a.rec[e0 + i] = d_mul(d_mul(p[i], a.step), r);
        }
        if (a.idx) {
#pragma unroll
            for (int i = 0; i < 8; ++i) a.idx[e0 + i] = (int16_t)(long long)d_mul(p[i], 2.0);
        }
    }
}

// Warp-per-groups kernel for power-of-two groups <= 256 (all reference uses):
// no shared memory, 16-byte loads and stores, numpy-order group sums via
// shuffles.  Phase 2 re-reads the group as 8-vectors (L1 hits).
template <typename TIn, int G>
__global__ void __launch_bounds__(256, 3) e8_warp_kernel(E8Args a) {
    using W = WarpGroup<G>;
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t e_base = warp * W::GPW * int64_t(G);          // first element of the warp
    const TIn *A = static_cast<const TIn *>(a.A);
    auto get = [&](int i) -> double {
        const int64_t e = e_base + i;
        return e < a.size ? double(__ldg(A + e)) : 0.0;
    };
    const double ss = warp_group_sumsq<G, double>(get);
    const double rms = d_add(sqrt(ss / double(G)), 1e-12);
    if (a.rms_out && (lane % W::LPG) == 0) {
        const int64_t g = e_base / G + lane / W::LPG;
        if (g * G < a.size) a.rms_out[g] = rms;
    }
    if (!a.rec && !a.idx) return;
    // approximation only (screen); a scale below 2^-100 disables the screen
    // (fp32 subnormal inputs would no longer meet the error bound)
    const double rs = d_mul(rms, a.step);
    const float inv_g = rs >= 0x1p-100 ? float(1.0 / rs) : __int_as_float(0x7fc00000);
    for (int vb = 0; vb < W::VPW; vb += 32) {
        const int vv = vb + lane;
        const int gg = (vv < W::VPW ? vv : W::VPW - 1) / W::VPG;
        const double r = __shfl_sync(0xffffffffu, rms, gg * W::LPG);
        const float inv = __shfl_sync(0xffffffffu, inv_g, gg * W::LPG);
        if (vv >= W::VPW) continue;
        const int64_t e0 = e_base + 8 * int64_t(vv);
        if (e0 >= a.size) continue;
        double y[8], p[8];
        const bool full8 = e0 + 8 <= a.size;
        if (sizeof(TIn) == 8 && full8 && ((reinterpret_cast<uintptr_t>(A + e0) & 15) == 0)) {
            const double2 *q = reinterpret_cast<const double2 *>(A + e0);
#pragma unroll
            for (int i = 0; i < 4; ++i) { const double2 t = __ldg(q + i); y[2 * i] = t.x; y[2 * i + 1] = t.y; }
        } else if (sizeof(TIn) == 4 && full8 && ((reinterpret_cast<uintptr_t>(A + e0) & 15) == 0)) {
            const float4 *q = reinterpret_cast<const float4 *>(A + e0);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const float4 t = __ldg(q + i);
                y[4 * i] = t.x; y[4 * i + 1] = t.y; y[4 * i + 2] = t.z; y[4 * i + 3] = t.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = e0 + i < a.size ? double(__ldg(A + e0 + i)) : 0.0;
        }
        // fp32 screen: y32 = RN32(g) * RN32(1 / (rms * step)), |y32 - y| <= |y32| 2^-22.3
        float y32[8];
        float ymax = 0.f;
        bool fin = true;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            y32[i] = __fmul_rn(float(y[i]), inv);
            ymax = fmaxf(ymax, fabsf(y32[i]));
            fin &= isfinite(y32[i]);
        }
        const float M = __fadd_rn(__fmul_rn(ymax, 0x1p-21f), 0x1p-40f);
        bool zero = true;
#pragma unroll
        for (int i = 0; i < 8; ++i) zero &= y[i] == 0.0;
        if (zero) {
            // y = (+-0 / rms) / step = +-0 exactly: the decode keeps each zero
            // (D8 point 0, coset point at distance 2 > 0)
#pragma unroll
            for (int i = 0; i < 8; ++i) p[i] = y[i];
        } else if (!(fin && ymax < 0x1p20f && e8_screen(y32, M, p))) {
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = (y[i] / r) / a.step;
            e8_point(y, p);
        }
        if (a.rec) {
            double o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = d_mul(d_mul(p[i], a.step), r);
            if (full8 && ((reinterpret_cast<uintptr_t>(a.rec + e0) & 15) == 0)) {
                double2 *q = reinterpret_cast<double2 *>(a.rec + e0);
#pragma unroll
                for (int i = 0; i < 4; ++i) q[i] = make_double2(o[2 * i], o[2 * i + 1]);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) if (e0 + i < a.size) a.rec[e0 + i] = o[i];
            }
        }
        if (a.idx) {
            short o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = (short)(long long)d_mul(p[i], 2.0);
            if ((reinterpret_cast<uintptr_t>(a.idx + e0) & 15) == 0) {
                int4 pk;
                pk.x = (unsigned short)o[0] | ((unsigned)(unsigned short)o[1] << 16);
                pk.y = (unsigned short)o[2] | ((unsigned)(unsigned short)o[3] << 16);
                pk.z = (unsigned short)o[4] | ((unsigned)(unsigned short)o[5] << 16);
                pk.w = (unsigned short)o[6] | ((unsigned)(unsigned short)o[7] << 16);
                *reinterpret_cast<int4 *>(a.idx + e0) = pk;
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) a.idx[e0 + i] = o[i];
            }
        }
    }
}

// ---- tensor-map form (fp64 input and output, groups of 256) ------------------
// Persistent warps walk 512-element chunks (two groups).  A warp's next chunk
// is loaded by a tensor-map copy (4 KB, 128-byte swizzled lines) into the
// second of its two shared buffers while it quantizes the current one; group
// sums read the chunk in numpy's chain order, 8-vectors are read and their
// reconstructions written back with conflict-free 16-byte accesses, and the
// chunk leaves by a tensor-map store.  Same arithmetic as e8_warp_kernel.
__device__ int g_e8_timeout = 0;

constexpr int kE8ChunkBytes = 4096;

__global__ void __launch_bounds__(256, 2)
e8_tma_kernel(const __grid_constant__ CUtensorMap tin, const __grid_constant__ CUtensorMap tout, E8Args a,
              int64_t nchunks) {
    using W = WarpGroup<256>;
    extern __shared__ __align__(1024) unsigned char e8_smem_raw[];
    __shared__ __align__(8) unsigned long long bars[8][2];
    unsigned char *sm = e8_smem_raw + ((1024u - (unsigned(__cvta_generic_to_shared(e8_smem_raw)) & 1023u)) & 1023u);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned buf0 = unsigned(__cvta_generic_to_shared(sm)) + unsigned(warp * 2 * kE8ChunkBytes);
    const unsigned bar0 = unsigned(__cvta_generic_to_shared(&bars[warp][0]));
    const int64_t nwarps = int64_t(gridDim.x) * 8;
    int64_t c = int64_t(blockIdx.x) * 8 + warp;
    if (lane == 0) {
        uq::tma::mbar_init(bar0, 1);
        uq::tma::mbar_init(bar0 + 8, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (c < nchunks) {
            uq::tma::mbar_arrive_expect_tx(bar0, kE8ChunkBytes);
            uq::tma::load2d(buf0, &tin, 0, int(32 * c), bar0);
        }
    }
    __syncwarp();
    bool fail = false;
    for (int k = 0; c < nchunks; c += nwarps, ++k) {
        const unsigned buf = buf0 + unsigned((k & 1) * kE8ChunkBytes);
        if (lane == 0 && c + nwarps < nchunks) {
            uq::tma::bulk_wait_read0();   // the store that last used the other buffer has read it
            const unsigned nb = bar0 + 8u * unsigned((k + 1) & 1);
            uq::tma::mbar_arrive_expect_tx(nb, kE8ChunkBytes);
            uq::tma::load2d(buf0 + unsigned(((k + 1) & 1) * kE8ChunkBytes), &tin, 0, int(32 * (c + nwarps)), nb);
        }
        uq::tma::mbar_wait_bounded(bar0 + 8u * unsigned(k & 1), unsigned((k >> 1) & 1), fail, &g_e8_timeout);
        auto get = [&](int i) -> double { return uq::tma::lds64d(buf + uq::tma::swz128<double>(i)); };
        const double ss = warp_group_sumsq<256, double>(get);
        const double rms = d_add(sqrt(ss / 256.0), 1e-12);
        const int64_t e_base = c * 512;
        if (a.rms_out && (lane % W::LPG) == 0) a.rms_out[e_base / 256 + lane / W::LPG] = rms;
        const double rs = d_mul(rms, a.step);
        const float inv_g = rs >= 0x1p-100 ? float(1.0 / rs) : __int_as_float(0x7fc00000);
#pragma unroll
        for (int vb = 0; vb < 64; vb += 32) {
            const int vv = vb + lane;                 // vector of the chunk
            const int gg = vv / W::VPG;
            const double r = __shfl_sync(0xffffffffu, rms, gg * W::LPG);
            const float inv = __shfl_sync(0xffffffffu, inv_g, gg * W::LPG);
            const int ln = vv >> 1, h = vv & 1;
            unsigned addr[4];
            double y[8], p[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                addr[q] = buf + unsigned(ln * 128 + (((4 * h + q) ^ (ln & 7)) << 4));
                const double2 t = uq::tma::lds128d(addr[q]);
                y[2 * q] = t.x;
                y[2 * q + 1] = t.y;
            }
            float y32[8];
            float ymax = 0.f;
            bool fin = true, zero = true;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                y32[i] = __fmul_rn(float(y[i]), inv);
                ymax = fmaxf(ymax, fabsf(y32[i]));
                fin &= isfinite(y32[i]);
                zero &= y[i] == 0.0;
            }
            const float M = __fadd_rn(__fmul_rn(ymax, 0x1p-21f), 0x1p-40f);
            if (zero) {
#pragma unroll
                for (int i = 0; i < 8; ++i) p[i] = y[i];
            } else if (!(fin && ymax < 0x1p20f && e8_screen(y32, M, p))) {
#pragma unroll
                for (int i = 0; i < 8; ++i) y[i] = (y[i] / r) / a.step;
                e8_point(y, p);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
                uq::tma::sts128d(addr[q], d_mul(d_mul(p[2 * q], a.step), r), d_mul(d_mul(p[2 * q + 1], a.step), r));
            if (a.idx) {
                short o[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = (short)(long long)d_mul(p[i], 2.0);
                int4 pk;
                pk.x = (unsigned short)o[0] | ((unsigned)(unsigned short)o[1] << 16);
                pk.y = (unsigned short)o[2] | ((unsigned)(unsigned short)o[3] << 16);
                pk.z = (unsigned short)o[4] | ((unsigned)(unsigned short)o[5] << 16);
                pk.w = (unsigned short)o[6] | ((unsigned)(unsigned short)o[7] << 16);
                *reinterpret_cast<int4 *>(a.idx + e_base + 8 * vv) = pk;
            }
        }
        uq::tma::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
            uq::tma::store2d(&tout, 0, int(32 * c), buf);
            uq::tma::bulk_commit();
        }
        __syncwarp();
    }
    if (lane == 0) uq::tma::bulk_wait0();
}

// Uses the tensor-map form for the whole 512-element chunks when it applies
// (fp64 in / out, group 256, 16-byte aligned rec and idx); returns the number
// of elements it covered (the rest goes to e8_warp_kernel), or -1 on error.
int64_t launch_e8_tma(const E8Args &a, cudaStream_t st) {
    if (a.group != 256 || !a.rec || (reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.rec) & 15) ||
        (a.idx && (reinterpret_cast<uintptr_t>(a.idx) & 15)) || !uq::tma::encode_fn())
        return 0;
    const int64_t nchunks = a.size / 512;
    if (nchunks < 1 || nchunks * 32 > (int64_t(1) << 31)) return 0;
    CUtensorMap mi, mo;
    const cuuint64_t dims[2] = {16, cuuint64_t(nchunks * 32)};
    const cuuint64_t strides[1] = {128};
    const cuuint32_t box[2] = {16, 32};
    if (!uq::tma::encode_lines(&mi, true, 2, a.A, dims, strides, box) ||
        !uq::tma::encode_lines(&mo, true, 2, a.rec, dims, strides, box))
        return 0;
    const size_t smem = size_t(8) * 2 * kE8ChunkBytes + 1024;
    if (uq::set_smem_attr(reinterpret_cast<const void *>(e8_tma_kernel), int(smem)) != cudaSuccess) {
        uq::check_cuda("e8 tma: set smem attribute");
        return -1;
    }
    int per_sm = 0;
    if (uq::occupancy_blocks(&per_sm, reinterpret_cast<const void *>(e8_tma_kernel), 256, smem) != cudaSuccess || per_sm < 1) {
        uq::check_cuda("e8 tma: occupancy");
        return -1;
    }
    const int64_t blocks = std::min<int64_t>((nchunks + 7) / 8, int64_t(per_sm) * uq::num_sms());
    { uq::ProfScope _p("e8_quant", st); e8_tma_kernel<<<unsigned(blocks), 256, smem, st>>>(mi, mo, a, nchunks); }
    if (uq::check_cuda("e8_tma_kernel launch") != UQ_OK) return -1;
    return nchunks * 512;
}

template <typename TIn, int G>
int launch_e8_warp(const E8Args &a, cudaStream_t st) {
    using W = WarpGroup<G>;
    const int64_t groups = (a.size + G - 1) / G;
    const int64_t warps = (groups + W::GPW - 1) / W::GPW;
    const int64_t blocks = (warps + 7) / 8;
    if (blocks > 0) { uq::ProfScope _p("e8_quant", st); e8_warp_kernel<TIn, G><<<unsigned(blocks), 256, 0, st>>>(a); }
    return uq::check_cuda("e8_warp_kernel launch");
}

template <typename TIn>
int dispatch_e8_warp(const E8Args &a, cudaStream_t st) {
    switch (a.group) {
        case 8: return launch_e8_warp<TIn, 8>(a, st);
        case 16: return launch_e8_warp<TIn, 16>(a, st);
        case 32: return launch_e8_warp<TIn, 32>(a, st);
        case 64: return launch_e8_warp<TIn, 64>(a, st);
        case 128: return launch_e8_warp<TIn, 128>(a, st);
        case 256: return launch_e8_warp<TIn, 256>(a, st);
    }
    return -1;
}

int e8_tile_elems(int group) {
    if (group >= 2048) return group;
    int t = group;
    while (t < 2048) t += group;
    // keep tile a multiple of 8 vectors' worth of threads
    return t;
}

template <typename TIn>
int launch_e8_quant(const E8Args &a0, cudaStream_t st) {
    if (sizeof(TIn) == 8) {
        const int64_t done = launch_e8_tma(a0, st);
        if (done < 0) return UQ_ERR_CUDA;
        if (done == a0.size) return UQ_OK;
        if (done > 0) {
            // the tail (less than one chunk; whole groups) through the warp kernel
            E8Args t = a0;
            t.A = static_cast<const double *>(a0.A) + done;
            t.size = a0.size - done;
            t.rec = a0.rec + done;
            if (a0.idx) t.idx = a0.idx + done;
            if (a0.rms_out) t.rms_out = a0.rms_out + done / 256;
            return dispatch_e8_warp<TIn>(t, st);
        }
    }
    {
        const int rc = dispatch_e8_warp<TIn>(a0, st);
        if (rc >= 0) return rc;
    }
    E8Args a = a0;
    a.tile = e8_tile_elems(a.group);
    const int ng = a.tile / a.group;
    const size_t smem = sizeof(double) * (size_t(a.tile) + ng + size_t(ng) * 32);
    const int threads = std::min(1024, std::max(32, ((a.tile / 8 + 31) / 32) * 32));
    const int64_t padded = (a.size + a.group - 1) / a.group * a.group;
    const int64_t grid = (padded + a.tile - 1) / a.tile;
    auto kern = e8_quant_kernel<TIn>;
    if (uq::set_smem_attr(reinterpret_cast<const void *>(kern), int(smem)) != cudaSuccess)
        return uq::check_cuda("e8: set smem attribute");
    if (grid > 0) { uq::ProfScope _p("e8_quant", st); kern<<<unsigned(grid), threads, smem, st>>>(a); }
    return uq::check_cuda("e8_quant_kernel launch");
}

// ---- q_uniform (qlab.py:100-106) ------------------------------------------------
// Per block of bs consecutive values: amax = max|x| + 1e-12 (in the array's
// dtype), xh = rint(x / amax * lvl) / lvl * amax, each step one IEEE operation
// in that dtype.  One warp per block.
template <typename T>
__global__ void q_uniform_kernel(const T *A, int64_t nblocks, int64_t bs, T lvl, T *out) {
    const int lane = threadIdx.x & 31;
    const int64_t w0 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t b = w0; b < nblocks; b += nw) {
        const T *x = A + b * bs;
        T m = T(0);
        for (int64_t i = lane; i < bs; i += 32) m = fmax(m, fabs(__ldg(x + i)));
        for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        const T amax = m + T(1e-12);
        for (int64_t i = lane; i < bs; i += 32) {
            const T q = rint((__ldg(x + i) / amax) * lvl);
            out[b * bs + i] = (q / lvl) * amax;
        }
    }
}

// ---- entropy of lattice indices --------------------------------------------
// Key: byte i = (2*p_i truncated) + 128, coordinate values must lie in
// [-127, 127]; byte 0 never occurs, so key 0 marks an empty slot.
__device__ __forceinline__ unsigned long long mix64(unsigned long long k) {
    k ^= k >> 33; k *= 0xff51afd7ed558ccdull; k ^= k >> 33; k *= 0xc4ceb9fe1a85ec53ull; k ^= k >> 33;
    return k;
}

template <typename Src>
__global__ void hash_count_kernel(Src src, int64_t nvec, unsigned long long *keys, unsigned *cnt,
                                  unsigned long long mask, int *overflow) {
    for (int64_t v = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; v < nvec;
         v += int64_t(gridDim.x) * blockDim.x) {
        unsigned long long key = 0;
        bool bad = false;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const long long c = src(v, i);
            bad |= (c < -127 || c > 127);
            key |= (unsigned long long)(c + 128) << (8 * i);
        }
        if (bad) { atomicExch(overflow, 1); continue; }
        unsigned long long h = mix64(key) & mask;
        for (unsigned long long probe = 0; probe <= mask; ++probe) {
            const unsigned long long prev = atomicCAS(keys + h, 0ull, key);
            if (prev == 0ull || prev == key) { atomicAdd(cnt + h, 1u); break; }
            h = (h + 1) & mask;
        }
    }
}

struct PtsSrc {  // (pts * 2).astype(int64) of an fp64 (nvec, 8) array
    const double *p;
    __device__ long long operator()(int64_t v, int i) const { return (long long)d_mul(__ldg(p + 8 * v + i), 2.0); }
};

// Per-CTA fixed-point sums of -p log2 p (p = cnt / total), 2^-64 units.
__global__ void entropy_partial_kernel(const unsigned *cnt, int64_t slots, double total,
                                       unsigned long long *part_hi, unsigned long long *part_lo) {
    __shared__ unsigned __int128 red[256];
    unsigned __int128 acc = 0;
    for (int64_t s = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; s < slots;
         s += int64_t(gridDim.x) * blockDim.x) {
        const unsigned c = cnt[s];
        if (c) {
            const double p = double(c) / total;
            const double t = -(p * log2(p));            // in [0, 0.531]
            acc += (unsigned __int128)(unsigned long long)(t * 18446744073709551616.0);  // * 2^64 < 2^63
        }
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        part_hi[blockIdx.x] = (unsigned long long)(red[0] >> 64);
        part_lo[blockIdx.x] = (unsigned long long)red[0];
    }
}

__global__ void entropy_final_kernel(const unsigned long long *hi, const unsigned long long *lo, int parts,
                                     double *bpw, const int *overflow) {
    unsigned __int128 s = 0;
    for (int i = 0; i < parts; ++i) s += ((unsigned __int128)hi[i] << 64) | lo[i];
    const double v = double((unsigned long long)(s >> 64)) + double((unsigned long long)s) * 5.421010862427522e-20;
    *bpw = (*overflow) ? -1.0 : v / 8.0;
}

constexpr int kEntParts = 296;

struct EntWs {
    unsigned long long *keys, *hi, *lo;
    unsigned *cnt;
    int *overflow;
    unsigned long long mask;
};

size_t entropy_ws_bytes(int64_t nvec, EntWs *w, void *base) {
    unsigned long long slots = 1024;
    while (slots < (unsigned long long)(2 * nvec)) slots <<= 1;
    uq::Carver c(base, ~size_t(0));
    EntWs t;
    t.keys = c.take<unsigned long long>(slots);
    t.cnt = c.take<unsigned>(slots);
    t.hi = c.take<unsigned long long>(kEntParts);
    t.lo = c.take<unsigned long long>(kEntParts);
    t.overflow = c.take<int>(1);
    t.mask = slots - 1;
    if (w) *w = t;
    return c.off;
}

template <typename Src>
int entropy_run(Src src, int64_t nvec, double *bpw, void *ws, size_t ws_bytes, cudaStream_t st) {
    EntWs w;
    const size_t need = entropy_ws_bytes(nvec, &w, ws);
    if (ws_bytes < need) return uq::fail(UQ_ERR_WORKSPACE, "entropy: workspace %zu < %zu", ws_bytes, need);
    const size_t slots = size_t(w.mask) + 1;
    cudaMemsetAsync(w.keys, 0, slots * sizeof(unsigned long long), st);
    cudaMemsetAsync(w.cnt, 0, slots * sizeof(unsigned), st);
    cudaMemsetAsync(w.overflow, 0, sizeof(int), st);
    const int grid = std::max(1, std::min<int>(int((nvec + 255) / 256), uq::num_sms() * 8));
    if (nvec > 0) { uq::ProfScope _p("hash_count", st); hash_count_kernel<<<grid, 256, 0, st>>>(src, nvec, w.keys, w.cnt, w.mask, w.overflow); }
    { uq::ProfScope _p("entropy_partial", st); entropy_partial_kernel<<<kEntParts, 256, 0, st>>>(w.cnt, int64_t(slots), double(nvec), w.hi, w.lo); }
    { uq::ProfScope _p("entropy_final", st); entropy_final_kernel<<<1, 1, 0, st>>>(w.hi, w.lo, kEntParts, bpw, w.overflow); }
    return uq::check_cuda("entropy kernels");
}

// ---- calibration (qlab.py:171-180) ------------------------------------------
// gather the subsampled, normalised vectors: sub[i] = x[8*pick[i] ..] / rms[group]
template <typename TIn>
__global__ void gather_gn_kernel(const TIn *A, int64_t size, int group, const double *rms,
                                 const int64_t *pick, int64_t ns, double *sub) {
    for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < ns * 8;
         t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t v = pick[t >> 3];
        const int64_t e = 8 * v + (t & 7);
        const double x = e < size ? double(__ldg(A + e)) : 0.0;
        sub[t] = x / rms[e / group];
    }
}

__global__ void e8_scaled_keys_kernel(const double *sub, int64_t ns, double step, double *pts) {
    for (int64_t v = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; v < ns;
         v += int64_t(gridDim.x) * blockDim.x) {
        double y[8], p[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = sub[8 * v + i] / step;
        e8_point(y, p);
#pragma unroll
        for (int i = 0; i < 8; ++i) pts[8 * v + i] = p[i];
    }
}

}  // namespace

namespace uq {
// Reads and clears the timeout flag of the tensor-map quantizer's bounded waits
// (after the caller synchronised); -1 on a CUDA error.
int e8_take_timeout() {
    int flag = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&flag, g_e8_timeout, sizeof(int)) != cudaSuccess) return -1;
    if (flag && cudaMemcpyToSymbol(g_e8_timeout, &zero, sizeof(int)) != cudaSuccess) return -1;
    return flag;
}

// Sets the flag as a timed-out wait would (host-side fault injection).
int e8_set_timeout() {
    const int one = 1;
    return cudaMemcpyToSymbol(g_e8_timeout, &one, sizeof(int)) == cudaSuccess ? 0 : -1;
}

int e8_quant(const void *A, int a_dtype, int64_t size, int64_t group, double step, double *rec,
             int16_t *idx, double *rms_out, cudaStream_t st) {
    NvtxRange _r("e8_quant");
    E8Args a{};
    a.A = A; a.size = size; a.group = int(group); a.step = step; a.rec = rec; a.idx = idx; a.rms_out = rms_out;
    if (a_dtype == UQ_F64) return launch_e8_quant<double>(a, st);
    if (a_dtype == UQ_F32) return launch_e8_quant<float>(a, st);
    return fail(UQ_ERR_INVALID, "e8: bad dtype");
}
}  // namespace uq

static int e8_check(int64_t size, int64_t group, const char *who) {
    if (size < 0) return uq::fail(UQ_ERR_INVALID, "%s: negative size", who);
    if (group < 8 || group % 8 != 0 || group > 8192)
        return uq::fail(UQ_ERR_UNSUPPORTED, "%s: group %lld must be a multiple of 8 in [8, 8192]", who, (long long)group);
    return UQ_OK;
}

extern "C" {

int uq_d8_decode(const double *Y, int64_t nvec, double *out, void *stream) {
    if (nvec < 0) return uq::fail(UQ_ERR_INVALID, "uq_d8_decode: nvec < 0");
    if (nvec == 0) return UQ_OK;
    if (!Y || !out) return uq::fail(UQ_ERR_INVALID, "uq_d8_decode: null pointer");
    const int grid = std::max(1, std::min<int>(int((nvec + 255) / 256), uq::num_sms() * 16));
    { uq::ProfScope _p("d8_decode", UQ_STREAM(stream)); d8_kernel<<<grid, 256, 0, UQ_STREAM(stream)>>>(Y, nvec, out, 0); }
    return uq::check_cuda("d8_kernel launch");
}

int uq_e8_decode(const double *Y, int64_t nvec, double *out, void *stream) {
    if (nvec < 0) return uq::fail(UQ_ERR_INVALID, "uq_e8_decode: nvec < 0");
    if (nvec == 0) return UQ_OK;
    if (!Y || !out) return uq::fail(UQ_ERR_INVALID, "uq_e8_decode: null pointer");
    const int grid = std::max(1, std::min<int>(int((nvec + 255) / 256), uq::num_sms() * 16));
    { uq::ProfScope _p("e8_decode", UQ_STREAM(stream)); d8_kernel<<<grid, 256, 0, UQ_STREAM(stream)>>>(Y, nvec, out, 1); }
    return uq::check_cuda("e8 decode launch");
}

int uq_e8_quant(const void *A, int a_dtype, int64_t size, int64_t group, double step, double *rec,
                int16_t *idx, void *stream) {
    int rc = e8_check(size, group, "uq_e8_quant");
    if (rc) return rc;
    if (!uq::dtype_size(a_dtype)) return uq::fail(UQ_ERR_INVALID, "uq_e8_quant: bad dtype");
    if (size == 0) return UQ_OK;
    if (!A || (!rec && !idx)) return uq::fail(UQ_ERR_INVALID, "uq_e8_quant: null pointer");
    return uq::e8_quant(A, a_dtype, size, group, step, rec, idx, nullptr, UQ_STREAM(stream));
}

size_t uq_e8_entropy_workspace_bytes(int64_t nvec) { return entropy_ws_bytes(nvec < 0 ? 0 : nvec, nullptr, nullptr); }

int uq_e8_entropy_bpw(const double *pts, int64_t nvec, double *bpw, void *workspace,
                      size_t workspace_bytes, void *stream) {
    if (nvec < 1) return uq::fail(UQ_ERR_INVALID, "uq_e8_entropy_bpw: need at least one vector");
    if (!pts || !bpw || !workspace) return uq::fail(UQ_ERR_INVALID, "uq_e8_entropy_bpw: null pointer");
    return entropy_run(PtsSrc{pts}, nvec, bpw, workspace, workspace_bytes, UQ_STREAM(stream));
}


int uq_e8_sample_indices(int64_t nvec, int64_t ns, int64_t *out_host) {
    if (nvec < 1 || ns < 0 || (ns > 0 && !out_host))
        return uq::fail(UQ_ERR_INVALID, "uq_e8_sample_indices: bad arguments (nvec=%lld ns=%lld)", (long long)nvec,
                        (long long)ns);
    uq::MT19937 g;
    g.seed(0);
    g.randint(0, nvec, ns, out_host);
    return UQ_OK;
}

size_t uq_e8_sample_gn_workspace_bytes(int64_t size, int64_t group) {
    if (size < 0 || group < 8) return 0;
    return uq::align_up(size_t((size + group - 1) / group) * 8, 256);
}

int uq_e8_sample_gn(const void *A, int a_dtype, int64_t size, int64_t group, const int64_t *vec_ids, int64_t count,
                    double *out, void *workspace, size_t workspace_bytes, void *stream) {
    int rc = e8_check(size, group, "uq_e8_sample_gn");
    if (rc) return rc;
    if (count < 0 || !uq::dtype_size(a_dtype)) return uq::fail(UQ_ERR_INVALID, "uq_e8_sample_gn: bad arguments");
    if (count == 0 || size == 0) return UQ_OK;
    if (!A || !vec_ids || !out || !workspace) return uq::fail(UQ_ERR_INVALID, "uq_e8_sample_gn: null pointer");
    if (workspace_bytes < uq_e8_sample_gn_workspace_bytes(size, group))
        return uq::fail(UQ_ERR_WORKSPACE, "uq_e8_sample_gn: workspace %zu too small", workspace_bytes);
    const cudaStream_t st = UQ_STREAM(stream);
    double *rms = static_cast<double *>(workspace);
    if ((rc = uq::e8_quant(A, a_dtype, size, group, 1.0, nullptr, nullptr, rms, st))) return rc;
    const int grid = std::max(1, std::min<int>(int((count * 8 + 255) / 256), uq::num_sms() * 16));
    uq::count_launch();
    if (a_dtype == UQ_F64)
        gather_gn_kernel<double><<<grid, 256, 0, st>>>(static_cast<const double *>(A), size, int(group), rms, vec_ids, count, out);
    else
        gather_gn_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float *>(A), size, int(group), rms, vec_ids, count, out);
    return uq::check_cuda("gather_gn_kernel launch");
}

size_t uq_e8_calibrate_sample_workspace_bytes(int64_t ns) {
    if (ns < 1) return 0;
    uq::Carver c(nullptr, ~size_t(0));
    c.take<double>(size_t(ns) * 8);
    c.take<double>(1);
    c.take<char>(entropy_ws_bytes(ns, nullptr, nullptr));
    return c.off;
}

int uq_e8_calibrate_sample(const double *sub, int64_t ns, double target_bpw, double *step_host, void *workspace,
                           size_t workspace_bytes, void *stream) {
    if (ns < 1 || !sub || !step_host || !workspace)
        return uq::fail(UQ_ERR_INVALID, "uq_e8_calibrate_sample: bad arguments");
    if (workspace_bytes < uq_e8_calibrate_sample_workspace_bytes(ns))
        return uq::fail(UQ_ERR_WORKSPACE, "uq_e8_calibrate_sample: workspace %zu too small", workspace_bytes);
    uq::Carver c(workspace, workspace_bytes);
    double *pts = c.take<double>(size_t(ns) * 8);
    double *bpw_d = c.take<double>(1);
    const size_t ent_bytes = entropy_ws_bytes(ns, nullptr, nullptr);
    void *ent = c.take<char>(ent_bytes);
    const cudaStream_t st = UQ_STREAM(stream);
    int rc;
    // qlab.py:174-180: 18 halvings of [0.3, 10] on the entropy of the decoded sample
    double lo = 0.3, hi = 10.0;
    for (int it = 0; it < 18; ++it) {
        const double mid = (lo + hi) / 2;
        const int g2 = std::max(1, std::min<int>(int((ns + 127) / 128), uq::num_sms() * 16));
        { uq::ProfScope _p("e8_scaled_keys", st); e8_scaled_keys_kernel<<<g2, 128, 0, st>>>(sub, ns, mid, pts); }
        if ((rc = uq::check_cuda("e8_scaled_keys_kernel launch"))) return rc;
        if ((rc = entropy_run(PtsSrc{pts}, ns, bpw_d, ent, ent_bytes, st))) return rc;
        double bpw = 0.0;
        if (cudaMemcpyAsync(&bpw, bpw_d, sizeof(double), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess)
            return uq::check_cuda("calibrate: read entropy");
        if (bpw < 0) return uq::fail(UQ_ERR_UNSUPPORTED, "calibrate: lattice index outside [-127, 127] at step %g", mid);
        if (bpw > target_bpw) lo = mid; else hi = mid;
    }
    *step_host = (lo + hi) / 2;
    return UQ_OK;
}

size_t uq_e8_calibrate_workspace_bytes(int64_t size, int64_t group) {
    if (size < 0 || group < 8) return 0;
    const int64_t padded = (size + group - 1) / group * group;
    const int64_t nvec = padded / 8, ns = nvec < 600000 ? nvec : 600000;
    uq::Carver c(nullptr, ~size_t(0));
    c.take<char>(uq_e8_sample_gn_workspace_bytes(size, group));
    c.take<int64_t>(size_t(ns));
    c.take<double>(size_t(ns) * 8);
    c.take<char>(uq_e8_calibrate_sample_workspace_bytes(ns));
    return c.off;
}

int uq_e8_calibrate(const void *A, int a_dtype, int64_t size, int64_t group, double target_bpw,
                    double *step_host, void *workspace, size_t workspace_bytes, void *stream) {
    int rc = e8_check(size, group, "uq_e8_calibrate");
    if (rc) return rc;
    if (size < 1 || !A || !step_host || !workspace || !uq::dtype_size(a_dtype))
        return uq::fail(UQ_ERR_INVALID, "uq_e8_calibrate: bad arguments");
    if (workspace_bytes < uq_e8_calibrate_workspace_bytes(size, group))
        return uq::fail(UQ_ERR_WORKSPACE, "uq_e8_calibrate: workspace %zu < %zu", workspace_bytes,
                        uq_e8_calibrate_workspace_bytes(size, group));
    const cudaStream_t st = UQ_STREAM(stream);
    const int64_t padded = (size + group - 1) / group * group;
    const int64_t nvec = padded / 8;
    const int64_t ns = nvec < 600000 ? nvec : 600000;
    uq::Carver c(workspace, workspace_bytes);
    const size_t gn_ws = uq_e8_sample_gn_workspace_bytes(size, group);
    void *gws = c.take<char>(gn_ws);
    int64_t *pick = c.take<int64_t>(size_t(ns));
    double *sub = c.take<double>(size_t(ns) * 8);
    const size_t cal_ws = uq_e8_calibrate_sample_workspace_bytes(ns);
    void *cws = c.take<char>(cal_ws);
    // RandomState(0).randint(0, nvec, ns) over the whole (padded) tensor
    std::vector<int64_t> h(static_cast<size_t>(ns), 0);
    if ((rc = uq_e8_sample_indices(nvec, ns, h.data()))) return rc;
    if (cudaMemcpyAsync(pick, h.data(), size_t(ns) * sizeof(int64_t), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return uq::check_cuda("calibrate: copy subsample indices");
    if ((rc = uq_e8_sample_gn(A, a_dtype, size, group, pick, ns, sub, gws, gn_ws, stream))) return rc;
    return uq_e8_calibrate_sample(sub, ns, target_bpw, step_host, cws, cal_ws, stream);
}

int uq_q_uniform(const void *A, int dtype, int64_t size, int64_t bs, int64_t lvl, void *out, void *stream) {
    if (size < 0 || bs < 1 || size % bs || !uq::dtype_size(dtype))
        return uq::fail(UQ_ERR_INVALID, "uq_q_uniform: cannot reshape array of size %lld into shape (-1,%lld)",
                        (long long)size, (long long)bs);
    if (size == 0) return UQ_OK;
    if (!A || !out) return uq::fail(UQ_ERR_INVALID, "uq_q_uniform: null pointer");
    const int64_t nblocks = size / bs;
    const int grid = int(std::max<int64_t>(1, std::min<int64_t>((nblocks + 7) / 8, int64_t(uq::num_sms()) * 16)));
    const cudaStream_t st = UQ_STREAM(stream);
    {
        uq::ProfScope _p("q_uniform", st);
        if (dtype == UQ_F64)
            q_uniform_kernel<double><<<grid, 256, 0, st>>>(static_cast<const double *>(A), nblocks, bs, double(lvl),
                                                           static_cast<double *>(out));
        else
            q_uniform_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float *>(A), nblocks, bs, float(lvl),
                                                          static_cast<float *>(out));
    }
    return uq::check_cuda("q_uniform_kernel launch");
}

}  // extern "C"
