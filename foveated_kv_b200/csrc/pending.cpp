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
FkvPromo* fkv_promo_create(int32_t, int32_t, int32_t, int32_t) {
    fkv::set_error("promotion pipeline: not implemented in this build");
    return nullptr;
}
int fkv_promo_register_archive(FkvPromo*, int32_t, const char*, const char*, int32_t, int32_t,
                               int32_t, int32_t, const int32_t*, int64_t) { return FKV_ERR_UNSUPPORTED; }
int fkv_promo_register_archive_host(FkvPromo*, int32_t, const uint16_t*, const uint16_t*, int32_t,
                                    int32_t, int32_t, int32_t, const int32_t*, int64_t) { return FKV_ERR_UNSUPPORTED; }
int fkv_promo_register_blob(FkvPromo*, int32_t, uint16_t*, uint16_t*, int32_t*, int32_t, int32_t,
                            int32_t, int32_t) { return FKV_ERR_UNSUPPORTED; }
int fkv_promo_drain(FkvPromo*, int32_t, const int32_t*, const int32_t*, const int32_t*, int32_t,
                    int32_t, int32_t, int32_t, int32_t) { return FKV_ERR_UNSUPPORTED; }
int fkv_promo_flush(FkvPromo*, void*, int32_t) { return FKV_ERR_UNSUPPORTED; }
int fkv_promo_stats(FkvPromo*, uint64_t*) { return FKV_ERR_UNSUPPORTED; }
int fkv_promo_stop(FkvPromo*) { return FKV_ERR_UNSUPPORTED; }
void fkv_promo_destroy(FkvPromo*) {}

}
