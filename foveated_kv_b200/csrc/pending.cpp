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

}
