// gk_random.cuh - device random draws for root noise (double precision).
//
// Gamma(alpha) by Marsaglia & Tsang (2000), "A simple method for generating
// gamma variables", with the alpha < 1 boost Gamma(alpha+1) * U^(1/alpha);
// standard normals by the Box-Muller transform. Uniforms come from PCG32
// (include/gk_common.h), 53 bits from two draws.
#pragma once

#include <cstdint>

#include "../../include/gk_common.h"

namespace gk {

__device__ __forceinline__ double uniform01(gk_pcg32& r) {
    const uint64_t hi = gk_pcg32_next(&r) >> 5, lo = gk_pcg32_next(&r) >> 6;  // 27 + 26 bits
    return ((double)(hi * 67108864ull + lo) + 0.5) * (1.0 / 9007199254740992.0);
}

__device__ __forceinline__ double normal01(gk_pcg32& r) {
    const double u1 = uniform01(r), u2 = uniform01(r);
    return sqrt(-2.0 * log(u1)) * cospi(2.0 * u2);
}

__device__ inline double gamma_draw(double alpha, gk_pcg32& r) {
    double boost = 1.0;
    if (alpha < 1.0) {
        boost = pow(uniform01(r), 1.0 / alpha);
        alpha += 1.0;
    }
    const double d = alpha - 1.0 / 3.0, c = 1.0 / sqrt(9.0 * d);
    for (int it = 0; it < 64; ++it) {
        const double x = normal01(r);
        double y = 1.0 + c * x;
        if (y <= 0.0) continue;
        y = y * y * y;
        const double u = uniform01(r);
        if (u < 1.0 - 0.0331 * x * x * x * x || log(u) < 0.5 * x * x + d * (1.0 - y + log(y))) return d * y * boost;
    }
    return d * boost;
}

// Max-normalised gamma draws over the legal actions of `root` that `allow`
// keeps (bit a & 31 of allow[a >> 5]) into out[82] (0 for the others), as
// GpuPUCT._search prepares them (python/kingdom_ai/gpu_puct.py:509-517).
__device__ inline void root_noise(const gk_bits& root, double alpha, gk_pcg32& r, float* out,
                                  const uint32_t* allow = nullptr) {
    const bool live = gk_reason(&root) == GK_NONE;
    gk_b96 placements = gk_b(0u, 0u, 0u);
    if (live && gk_stock(&root, gk_actor(&root)) > 0) {
        const gk_b96 occ = gk_or(gk_or(gk_get(&root, GK_PLANE_BLACK), gk_get(&root, GK_PLANE_WHITE)),
                                 gk_get(&root, GK_PLANE_NEUTRAL));
        const gk_b96 owned = gk_or(gk_get(&root, GK_PLANE_OWN_BLACK), gk_get(&root, GK_PLANE_OWN_WHITE));
        placements = gk_andnot(gk_andnot(gk_valid(), occ), owned);
    }
    double g[GK_ACTIONS];
    double largest = 0.0;
    for (int a = 0; a < GK_ACTIONS; ++a) {
        g[a] = 0.0;
        const bool legal = live && (a == GK_PASS || gk_test(placements, a + a / 9)) &&
                           (allow == nullptr || ((allow[a >> 5] >> (a & 31)) & 1u) != 0u);
        if (legal) {
            double x = gamma_draw(alpha, r);
            if (!isfinite(x) || x < 0.0) x = 0.0;
            g[a] = x;
            largest = fmax(largest, x);
        }
    }
    const double scale = largest > 2.2250738585072014e-308 ? largest : 2.2250738585072014e-308;
    for (int a = 0; a < GK_ACTIONS; ++a) out[a] = (float)(g[a] / scale);
}

}  // namespace gk
