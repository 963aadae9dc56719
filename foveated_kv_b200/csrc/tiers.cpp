// Host-side tier layout and error reporting for libfkv.
#include <algorithm>
#include <cstring>

#include "fkv_common.h"

namespace fkv {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

}  // namespace fkv

extern "C" {

int fkv_abi_version(void) { return 2; }

const char* fkv_last_error(void) { return fkv::g_last_error.c_str(); }

// Same integer arithmetic as MLXTierConfig.tier_boundaries
// (src/foveated_kv/mlx_foveated.py:128-169).  near_pct and the headroom
// fraction are doubles, like Python floats, so int(S * near_pct) truncates the
// same double product.
int fkv_tier_boundaries(int32_t S, double near_pct, int32_t n_sinks, int32_t window_size,
                        double promo_headroom_pct, int32_t promo_headroom_min,
                        FkvTierLayout* out) {
    FKV_REQUIRE(out != nullptr, FKV_ERR_INVALID, "fkv_tier_boundaries: out is NULL");
    FKV_REQUIRE(S >= 0 && n_sinks >= 0 && window_size >= 0 && promo_headroom_min >= 0,
                FKV_ERR_INVALID, "fkv_tier_boundaries: negative size (S=%d sinks=%d window=%d)",
                S, n_sinks, window_size);
    FKV_REQUIRE(near_pct >= 0.0 && near_pct <= 1.0 && promo_headroom_pct >= 0.0,
                FKV_ERR_INVALID, "fkv_tier_boundaries: near_pct=%g headroom_pct=%g out of range",
                near_pct, promo_headroom_pct);
    const int32_t ns = std::min(n_sinks, S);
    const int32_t window = std::min(window_size, std::max(S - ns, 0));
    const int32_t near_reserved = ns + window;
    int64_t R_total = std::max<int64_t>((int64_t)((double)S * near_pct), near_reserved);
    if (S - R_total < 0) R_total = S;
    const int32_t mid_start = ns;
    const int32_t mid_end = window > 0 ? S - window : S;
    const int32_t mid_len = std::max(mid_end - mid_start, 0);
    const int32_t near_from_mid =
        (int32_t)std::min<int64_t>(std::max<int64_t>(R_total - near_reserved, 0), mid_len);
    const int32_t R = ns + near_from_mid + window;
    const int32_t headroom =
        std::max((int32_t)((double)R * promo_headroom_pct), promo_headroom_min);
    out->S = S;
    out->n_sinks = ns;
    out->window = window;
    out->near_from_mid = near_from_mid;
    out->r_actual = R;
    out->n_near_padded = R + headroom;
    out->mid_start = mid_start;
    out->mid_end = mid_end;
    out->near_mid_start = mid_end - near_from_mid;
    out->far_count = out->near_mid_start - mid_start;
    return FKV_OK;
}

}  // extern "C"
