// E8 nearest-point decode on one 8-vector in registers (qlab.py:133-149):
// the exact fp64 Conway-Sloane decode and its fp32 screen with proven
// margins.  Shared by the q_e8_fast quantizer and the finite-codebook q_e8.
#pragma once
#include <cuda_runtime.h>

#include "uq_common.cuh"

namespace {

// ---- D8 / E8 decode on one vector in registers ------------------------------
__device__ __forceinline__ double sum8_pairwise(const double v[8]) {
    return d_add(d_add(d_add(v[0], v[1]), d_add(v[2], v[3])), d_add(d_add(v[4], v[5]), d_add(v[6], v[7])));
}

// qlab.py:133-142: round half to even; odd coordinate sum -> move the first
// coordinate of largest |error| by sign(error) (0 when the error is 0).
__device__ __forceinline__ void d8_point(const double y[8], double f[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = rint(y[i]);
    const long long s = (long long)sum8_pairwise(f);
    if (s % 2 != 0) {
        int k = 0;
        double best = fabs(d_sub(y[0], f[0]));
#pragma unroll
        for (int i = 1; i < 8; ++i) {
            const double a = fabs(d_sub(y[i], f[i]));
            if (a > best) { best = a; k = i; }
        }
        double ek = 0.0;
#pragma unroll
        for (int i = 0; i < 8; ++i) if (i == k) ek = d_sub(y[i], f[i]);
        const double sg = ek > 0.0 ? 1.0 : (ek < 0.0 ? -1.0 : 0.0);
#pragma unroll
        for (int i = 0; i < 8; ++i) if (i == k) f[i] = d_add(f[i], sg);
    }
}

// qlab.py:144-149
__device__ __forceinline__ void e8_point(const double y[8], double p[8]) {
    double a[8], b[8], ym[8], da[8], db[8];
    d8_point(y, a);
#pragma unroll
    for (int i = 0; i < 8; ++i) ym[i] = d_sub(y[i], 0.5);
    d8_point(ym, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        b[i] = d_add(b[i], 0.5);
        const double ea = d_sub(y[i], a[i]), eb = d_sub(y[i], b[i]);
        da[i] = d_mul(ea, ea);
        db[i] = d_mul(eb, eb);
    }
    const bool use_b = sum8_pairwise(db) < sum8_pairwise(da);
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = use_b ? b[i] : a[i];
}

// ---- screened decode ----------------------------------------------------------
// The lattice point p depends on y only through 16 roundings, two first-index
// argmax choices, two signs and one distance comparison.  The screen decodes
// an fp32 approximation y32 of y (|y32 - y| <= M) and accepts the point only
// if every one of those decisions holds with a margin larger than the
// approximation error; the point itself (integers / half-integers) is then
// exactly the fp64 decode's.  Anything closer than the margins goes to the
// exact fp64 path.  Margins, with |e| <= 1 for coordinate errors:
//   roundings: distance to the half-integer boundary > 2M + 2^-22
//   argmax:    largest |e| exceeds the second largest by > 2M + 2^-22
//   sign:      |e_k| > M + 2^-22
//   distances: |da - db| > 48 M + 2^-14 (8 terms, each off by <= 3M, plus
//              fp32 rounding of sums <= 18)
__device__ __forceinline__ bool d8_screen(const float y[8], float f[8], float M) {
    const float tr = 2.f * M + 0x1p-22f;
    float best = -1.f, second = -1.f;
    int k = 0;
    bool ok = true;
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        f[i] = rintf(y[i]);
        const float ae = fabsf(__fsub_rn(y[i], f[i]));
        ok &= __fsub_rn(0.5f, ae) > tr;
        if (ae > best) { second = best; best = ae; k = i; }
        else if (ae > second) second = ae;
        sum = __fadd_rn(sum, f[i]);
    }
    // odd coordinate sum: move coordinate k by sign(e_k).  Branch-free (the
    // parity differs between the lanes of a warp); even sums keep f as is.
    const bool odd = int(sum) & 1;
    float ek = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ek = i == k ? __fsub_rn(y[i], f[i]) : ek;
    ok &= !odd || (__fsub_rn(best, second) > tr && fabsf(ek) > M + 0x1p-22f);
    const float sg = ek > 0.f ? 1.f : -1.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = (odd && i == k) ? __fadd_rn(f[i], sg) : f[i];
    return ok;
}

__device__ __forceinline__ float sum8f(const float v[8]) {
    return __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3])),
                     __fadd_rn(__fadd_rn(v[4], v[5]), __fadd_rn(v[6], v[7])));
}

// Returns true and the E8 point of y (given as y32, |y32 - y| <= M) when the
// screen decides every step; false otherwise.
__device__ __forceinline__ bool e8_screen(const float y[8], float M, double p[8]) {
    float a[8], b[8], ym[8], da[8], db[8];
    bool ok = d8_screen(y, a, M);
#pragma unroll
    for (int i = 0; i < 8; ++i) ym[i] = __fsub_rn(y[i], 0.5f);
    ok &= d8_screen(ym, b, M + 0x1p-24f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        b[i] = __fadd_rn(b[i], 0.5f);
        const float ea = __fsub_rn(y[i], a[i]), eb = __fsub_rn(y[i], b[i]);
        da[i] = __fmul_rn(ea, ea);
        db[i] = __fmul_rn(eb, eb);
    }
    const float sa = sum8f(da), sb = sum8f(db);
    ok &= fabsf(__fsub_rn(sa, sb)) > __fadd_rn(__fmul_rn(48.f, M), 0x1p-14f);
    const bool use_b = sb < sa;
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = double(use_b ? b[i] : a[i]);
    return ok;
}

}  // namespace
