// Shared host-side helpers for libfkv: thread-local error string, checks.
#pragma once
#include <cstdarg>
#include <cstdio>
#include <string>

#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/fkv.h"

namespace fkv {

void set_error(const char* fmt, ...);
void clear_error();

// Batched promotion scatter (promo_scatter.cu): `stage` is a device copy of
// [K rows n*D | V rows n*D] fp16, destination rows n int64 (row index into
// near_k / near_v), then m (near_valid index, new count) int32 pairs.
int promo_scatter(const void* stage, int n, int m, int D, uint16_t* near_k, uint16_t* near_v,
                  int32_t* near_valid, cudaStream_t st);

}  // namespace fkv

#define FKV_REQUIRE(cond, code, ...)      \
    do {                                  \
        if (!(cond)) {                    \
            ::fkv::set_error(__VA_ARGS__); \
            return (code);                \
        }                                 \
    } while (0)

#define FKV_CUDA_CHECK(expr)                                                              \
    do {                                                                                  \
        cudaError_t _e = (expr);                                                          \
        if (_e != cudaSuccess) {                                                          \
            ::fkv::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e),      \
                             __FILE__, __LINE__);                                         \
            return FKV_ERR_CUDA;                                                          \
        }                                                                                 \
    } while (0)

#define FKV_LAUNCH_CHECK()                                                                \
    do {                                                                                  \
        cudaError_t _e = cudaGetLastError();                                              \
        if (_e != cudaSuccess) {                                                          \
            ::fkv::set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(_e),  \
                             __FILE__, __LINE__);                                         \
            return FKV_ERR_CUDA;                                                          \
        }                                                                                 \
    } while (0)
