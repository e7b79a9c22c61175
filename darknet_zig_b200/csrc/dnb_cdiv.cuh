// Division by a per-launch constant, correctly rounded without a division instruction per
// element: the element count of normalize_delta (blas.zig:200) in the fused batchnorm
// kernels and the standalone op.
#pragma once

#include "dnb_common.cuh"

namespace dnb {

// normalize_delta's division by the element count (blas.zig:200, `/ (spatial * batch)`), a
// constant of the launch, correctly rounded without a division instruction per element:
//     q = fma(v, zh, v * zl),  zh = RN(1/d), zl = RN(1/d - zh)
// (the division-by-a-known-divisor method of Brisebarre, Muller and Raina, IEEE Trans.
// Computers 53(8), 2004). The method is exact for most divisors but not all, so the host
// checks it for this divisor against IEEE division on every significand of one binade,
// [1, 2): scaling v by 2^k scales every intermediate and the exact quotient by 2^k, so the
// check covers every v whose intermediates stay normal, |v| >= lo. Other v (zero, tiny,
// infinite, NaN) and divisors that fail the check take a real IEEE division. A power of two
// needs neither: v * (1/d) is then v / d for every v.
struct ConstDiv {
    float d = 1.0f;       // the divisor
    float zh = 1.0f;      // RN(1/d)
    float zl = 0.0f;      // RN(1/d - zh)
    unsigned lo = 0u;     // bits of the smallest |v| the two-operation form serves (0x7f800000: none)
    int pow2 = 0;         // d is a power of two: v * zh is v / d for every v, no range test
};
// The descriptor of divisor d (verified once per significand of d and cached; thread-safe).
ConstDiv const_div(float d);

namespace {

// IEEE division, kept out of line so that the rare out-of-range numerators branch to it and
// the common path carries no division instructions
__device__ __noinline__ float div_ieee(float v, float d) { return v / d; }
__device__ __noinline__ float4 div4_ieee(float4 v, float d) {
    return make_float4(v.x / d, v.y / d, v.z / d, v.w / d);
}
// true when lo <= |v| <= FLT_MAX, compared as bits (NaN and inf fall outside)
__device__ __forceinline__ bool div_in_range(unsigned m, unsigned lo) { return m >= lo && m <= 0x7f7fffffu; }
__device__ __forceinline__ float div_const(float v, const ConstDiv &k) {
    if (k.pow2) return v * k.zh;
    const float q = __fmaf_rn(v, k.zh, v * k.zl);
    if (!div_in_range(__float_as_uint(v) & 0x7fffffffu, k.lo)) return div_ieee(v, k.d);
    return q;
}
// four at once: one range test (on the smallest and largest magnitude) and one branch
__device__ __forceinline__ float4 div4_const(float4 v, const ConstDiv &k) {
    if (k.pow2) return make_float4(v.x * k.zh, v.y * k.zh, v.z * k.zh, v.w * k.zh);
    const unsigned mx = __float_as_uint(v.x) & 0x7fffffffu, my = __float_as_uint(v.y) & 0x7fffffffu;
    const unsigned mz = __float_as_uint(v.z) & 0x7fffffffu, mw = __float_as_uint(v.w) & 0x7fffffffu;
    const unsigned lo = min(min(mx, my), min(mz, mw)), hi = max(max(mx, my), max(mz, mw));
    if (lo < k.lo || hi > 0x7f7fffffu) return div4_ieee(v, k.d);
    return make_float4(__fmaf_rn(v.x, k.zh, v.x * k.zl), __fmaf_rn(v.y, k.zh, v.y * k.zl),
                       __fmaf_rn(v.z, k.zh, v.z * k.zl), __fmaf_rn(v.w, k.zh, v.w * k.zl));
}
}  // namespace
}  // namespace dnb
