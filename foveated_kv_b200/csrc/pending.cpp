// Entry points declared in fkv.h whose implementation is not in this build
// yet: they fail loudly with FKV_ERR_UNSUPPORTED.
#include "fkv_common.h"

extern "C" {

size_t fkv_select_importance_workspace_bytes(const FkvTierLayout*, int32_t, int32_t, int32_t) {
    return 0;
}
int fkv_select_importance(const FkvTierLayout*, int32_t, int32_t, int32_t, int32_t,
                          const uint16_t*, int64_t, const uint16_t*, int32_t*, int32_t*, int32_t*,
                          void*, size_t, void*) {
    fkv::set_error("fkv_select_importance: not implemented in this build");
    return FKV_ERR_UNSUPPORTED;
}
int fkv_decode_turbo(const FkvDecodeShape*, const uint16_t*, const uint16_t*, const int32_t*,
                     const uint8_t*, const uint8_t*, const uint16_t*, const uint16_t*,
                     const uint8_t*, const uint16_t*, const float*, const float*, const float*,
                     const uint16_t*, const uint16_t*, const uint16_t*, uint16_t*, int32_t*,
                     int32_t*, void*, size_t, void*) {
    fkv::set_error("fkv_decode_turbo: not implemented in this build");
    return FKV_ERR_UNSUPPORTED;
}

}
