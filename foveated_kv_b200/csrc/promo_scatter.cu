// Device side of the batched promotion: one host->device copy brings a whole
// drain's worth of exact fp16 K/V rows (packed by the promotion worker in
// pinned memory) to the device; promo_rows_kernel writes each row into its
// near-tier headroom slot, and promo_counts_kernel, launched after it on the
// same stream, stores the new near_valid counts -- so a decode launch that
// reads a new count finds every row it covers in place (the reference's
// release fence before the near_valid bump, promotion_pipeline.cpp:233-238).
#include <cuda_runtime.h>

#include <cstdint>

#include "fkv_common.h"

namespace {

// one warp per promoted row: K row then V row, 16-byte vectors
__global__ void promo_rows_kernel(const uint16_t* __restrict__ src_k, const uint16_t* __restrict__ src_v,
                                  const int64_t* __restrict__ dst_row, int n, int D,
                                  uint16_t* __restrict__ near_k, uint16_t* __restrict__ near_v) {
    const int warp = (int)(blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32);
    const int lane = threadIdx.x & 31;
    if (warp >= n) return;
    const int vecs = D / 8;   // 16-byte vectors per row
    const int64_t dst = dst_row[warp] * D;
    const uint4* sk = reinterpret_cast<const uint4*>(src_k + (int64_t)warp * D);
    const uint4* sv = reinterpret_cast<const uint4*>(src_v + (int64_t)warp * D);
    uint4* dk = reinterpret_cast<uint4*>(near_k + dst);
    uint4* dv = reinterpret_cast<uint4*>(near_v + dst);
    for (int i = lane; i < 2 * vecs; i += 32) {
        if (i < vecs) dk[i] = sk[i];
        else dv[i - vecs] = sv[i - vecs];
    }
}

// (index, new count) pairs
__global__ void promo_counts_kernel(const int32_t* __restrict__ upd, int m, int32_t* __restrict__ near_valid) {
    const int i = (int)(blockIdx.x * blockDim.x + threadIdx.x);
    if (i < m) near_valid[upd[2 * i]] = upd[2 * i + 1];
}

}  // namespace

namespace fkv {

int promo_scatter(const void* stage, int n, int m, int D, uint16_t* near_k, uint16_t* near_v,
                  int32_t* near_valid, cudaStream_t st) {
    const auto* base = static_cast<const uint8_t*>(stage);
    const size_t rows = (size_t)n * D * sizeof(uint16_t);
    const auto* sk = reinterpret_cast<const uint16_t*>(base);
    const auto* sv = reinterpret_cast<const uint16_t*>(base + rows);
    const auto* dst = reinterpret_cast<const int64_t*>(base + 2 * rows);
    const auto* upd = reinterpret_cast<const int32_t*>(base + 2 * rows + (size_t)n * sizeof(int64_t));
    if (n > 0) {
        constexpr int kWarps = 8;
        promo_rows_kernel<<<(n + kWarps - 1) / kWarps, kWarps * 32, 0, st>>>(sk, sv, dst, n, D, near_k,
                                                                            near_v);
        FKV_LAUNCH_CHECK();
    }
    if (m > 0) {
        promo_counts_kernel<<<(m + 255) / 256, 256, 0, st>>>(upd, m, near_valid);
        FKV_LAUNCH_CHECK();
    }
    return FKV_OK;
}

}  // namespace fkv
