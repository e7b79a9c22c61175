// The host side of dnb_cdiv.cuh: the per-divisor check of the two-operation division.
#include <math.h>
#include <string.h>

#include <mutex>
#include <utility>
#include <vector>

#include "dnb_cdiv.cuh"

namespace dnb {

// Verifies q = fma(a, zh, a * zl) against IEEE division a / d for every a in [1, 2) on the
// host (float division and fmaf are correctly rounded there, as fma is on the device). The
// verdict depends only on the significand of d: scaling d by 2^k scales zh and zl by 2^-k.
// About 2^23 divisions, tens of milliseconds, once per significand and process.
ConstDiv const_div(float d) {
    ConstDiv k;
    k.d = d;
    k.lo = 0x7f800000u;  // no v takes the two-operation form until the check passes
    if (!(d >= 1.0f) || !(d <= 0x1p40f)) return k;  // counts; zh and zl stay normal
    k.zh = 1.0f / d;
    k.zl = (float)(1.0 / (double)d - (double)k.zh);
    int e2 = 0;
    if (frexpf(d, &e2) == 0.5f) {  // 1/d is exact
        k.pow2 = 1;
        k.zl = 0.0f;
        return k;
    }
    uint32_t dbits;
    memcpy(&dbits, &d, 4);
    const uint32_t key = dbits & 0x007fffffu;
    static std::mutex mu;
    static std::vector<std::pair<uint32_t, bool>> verdicts;
    int known = -1;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const auto &v : verdicts)
            if (v.first == key) known = v.second ? 1 : 0;
    }
    if (known < 0) {
        // the check runs on the divisor with the same significand in [1, 2)
        int e = 0;
        const float d1 = ldexpf(frexpf(d, &e), 1);
        const float zh1 = 1.0f / d1;
        const float zl1 = (float)(1.0 / (double)d1 - (double)zh1);
        bool ok = true;
        for (uint32_t m = 0; m < (1u << 23) && ok; ++m) {
            const uint32_t bits = 0x3f800000u | m;
            float a;
            memcpy(&a, &bits, 4);
            volatile float t = a * zl1;  // one rounding, as on the device (no contraction)
            const float q = fmaf(a, zh1, t);
            ok = q == a / d1;
        }
        std::lock_guard<std::mutex> lock(mu);
        verdicts.emplace_back(key, ok);
        known = ok ? 1 : 0;
    }
    if (!known) return k;
    // |v| from which every intermediate is normal: |v * zl| >= 2^-126 and |v / d| >= 2^-126
    // (factors of 2 for margin); below it, and for zero, v / d is divided
    float lo = ldexpf(d, -124);
    if (k.zl != 0.0f) lo = fmaxf(lo, ldexpf(1.0f, -125) / fabsf(k.zl));
    if (lo < 0x1p127f) memcpy(&k.lo, &lo, 4);
    return k;
}

}  // namespace dnb
