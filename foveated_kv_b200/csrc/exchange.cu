// Sequence-split exchange over NVLink peer memory, fused with the merge.
//
// Each rank of a sequence split holds one block of partial records
// ([N records of (m, l, min_near, max_far, o[D])] followed by N argmax
// values) after its partial decode.  fkv_exchange_combine replaces the
// all-gather + merge of that step with ONE kernel launch per rank:
//
//   1. every block copies its share of the local record block into slot
//      `rank` of every rank's receive buffer with plain stores to the peers'
//      memory (CUDA IPC mappings over NVLink; no TMA, no multicast);
//   2. the block that finishes the copies last (a counter in the rank's own
//      state words) publishes the step's sequence number in every rank's
//      flag for this rank (release, system scope);
//   3. every block waits (bounded, acquire) until all P flags of its own
//      receive buffer carry the step's sequence number, then merges the P
//      records of its output row n in rank order (earliest rank wins max_far
//      ties), as fkv_combine_partials does.
//
// Receive buffers are double-buffered by the parity of the sequence number:
// a rank can only start writing step t + 2 into a peer after its own step
// t + 1 merge, which waited for the peer's step t + 1 flag, which the peer
// wrote after finishing its step t merge -- so no slot is overwritten while
// it is read.  The sequence number lives in device memory (state[0]) and is
// advanced by the launch itself, so a captured step replays correctly.
//
// No counterpart in the reference (it has no multi-device code).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "decode_common.cuh"
#include "fkv_common.h"

using namespace fkvdev;

namespace {

constexpr int kExThreads = 128;
constexpr uint32_t kExSpinLimit = 1u << 23;   // x 32+ ns back-off: about half a second

__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Receive buffer of one rank: flags [2][P] int32 (padded to 64 bytes), then
// [2][P][stride] f32 record blocks.
__host__ __device__ inline size_t ex_flag_bytes(int P) { return ((size_t)2 * P * 4 + 63) & ~(size_t)63; }

template <int D>
__global__ void __launch_bounds__(kExThreads)
    exchange_combine_kernel(int P, int rank, int N, int64_t stride, const float* __restrict__ local,
                            const uint64_t* __restrict__ peers, uint8_t* __restrict__ mine,
                            int32_t* __restrict__ state, float margin, uint16_t* __restrict__ out,
                            int32_t* __restrict__ flags, int32_t* __restrict__ tokens) {
    const int n = blockIdx.x, tid = threadIdx.x;
    __shared__ int sh_seq;
    if (tid == 0) sh_seq = *reinterpret_cast<volatile int32_t*>(state) + 1;
    __syncthreads();
    const int seq = sh_seq, par = seq & 1;
    const size_t fb = ex_flag_bytes(P);
    // 1. this block's share of the local block -> slot `rank` of every rank
    const int64_t v4 = stride / 4;
    const float4* src = reinterpret_cast<const float4*>(local);
    for (int r = 0; r < P; ++r) {
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(peers[r]) + fb) +
                      ((int64_t)par * P + rank) * v4;
        for (int64_t i = (int64_t)n * kExThreads + tid; i < v4; i += (int64_t)gridDim.x * kExThreads)
            dst[i] = src[i];
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
        const int old = atomicAdd(state + 1, 1);
        if (old == (int)gridDim.x - 1) {
            state[1] = 0;
            __threadfence_system();
            for (int r = 0; r < P; ++r)
                st_release_sys(reinterpret_cast<int32_t*>(peers[r]) + par * P + rank, seq);
        }
    }
    // 2. wait for every rank's block of this step
    const int32_t* myflags = reinterpret_cast<const int32_t*>(mine) + par * P;
    if (tid < P) {
        uint32_t i = 0;
        while (ld_acquire_sys(myflags + tid) != seq) {
            if (++i > kExSpinLimit) {
                atomicExch(state + 3, FKV_ERR_TIMEOUT);
                break;
            }
            __nanosleep(32);
        }
    }
    __syncthreads();
    __threadfence();
    // 3. merge row n over the P blocks in rank order
    const float* blocks = reinterpret_cast<const float*>(mine + fb) + (int64_t)par * P * stride;
    const int64_t rs = D + 4;
    const int64_t argoff = (int64_t)N * rs;
    float M = -INFINITY;
    for (int k = 0; k < P; ++k) M = fmaxf(M, blocks[k * stride + n * rs]);
    for (int d = tid; d < D; d += kExThreads) {
        float L = 0.f, acc = 0.f;
        if (M != -INFINITY) {
            for (int k = 0; k < P; ++k) {
                const float* rec = blocks + k * stride + n * rs;
                if (rec[0] == -INFINITY) continue;
                const float wgt = exp2f((rec[0] - M) * kLog2e);
                L = fmaf(wgt, rec[1], L);
                acc = fmaf(wgt, rec[4 + d], acc);
            }
        }
        out[(int64_t)n * D + d] = __half_as_ushort(__float2half_rn(L > 0.f ? acc / L : 0.f));
    }
    if (tid == 0) {
        float mn = INFINITY, mf = -INFINITY;
        int af = -1;
        for (int k = 0; k < P; ++k) {
            const float* rec = blocks + k * stride + n * rs;
            mn = fminf(mn, rec[2]);
            if (rec[3] > mf) {   // rank order: the first rank with the strict max wins
                mf = rec[3];
                af = reinterpret_cast<const int32_t*>(blocks + k * stride + argoff)[n];
            }
        }
        flags[n] = (mf > mn + margin) ? 1 : 0;
        tokens[n] = af;
        // the last block to finish advances the sequence number for the next launch
        const int old = atomicAdd(state + 2, 1);
        if (old == (int)gridDim.x - 1) {
            state[2] = 0;
            state[0] = seq;
        }
    }
}

using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetRangeFn get_range_fn() {
    static GetRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q{};
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetRangeFn>(f);
    });
    return fn;
}

}  // namespace

extern "C" {

size_t fkv_exchange_recv_bytes(int32_t P, int32_t N, int32_t D) {
    if (P <= 0 || N <= 0 || (D != 64 && D != 128)) return 0;
    const int64_t stride = ((int64_t)N * (D + 4) + N + 3) & ~(int64_t)3;
    return ex_flag_bytes(P) + (size_t)2 * P * stride * sizeof(float);
}

int64_t fkv_exchange_block_stride(int32_t N, int32_t D) {
    return ((int64_t)N * (D + 4) + N + 3) & ~(int64_t)3;
}

int fkv_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int fkv_ipc_get_handle(const void* dev_ptr, uint8_t* handle, int64_t* offset) {
    fkv::clear_error();
    FKV_REQUIRE(dev_ptr && handle && offset, FKV_ERR_INVALID, "fkv_ipc_get_handle: NULL argument");
    GetRangeFn range = get_range_fn();
    FKV_REQUIRE(range != nullptr, FKV_ERR_CUDA, "cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    FKV_REQUIRE(range(&base, &size, (CUdeviceptr)dev_ptr) == CUDA_SUCCESS, FKV_ERR_CUDA,
                "cuMemGetAddressRange failed for %p", dev_ptr);
    cudaIpcMemHandle_t h;
    FKV_CUDA_CHECK(cudaIpcGetMemHandle(&h, (void*)base));
    std::memcpy(handle, &h, sizeof(h));
    *offset = (int64_t)((CUdeviceptr)dev_ptr - base);
    return FKV_OK;
}

int fkv_ipc_open(const uint8_t* handle, int64_t offset, void** dev_ptr) {
    fkv::clear_error();
    FKV_REQUIRE(handle && dev_ptr && offset >= 0, FKV_ERR_INVALID, "fkv_ipc_open: bad argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    FKV_CUDA_CHECK(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    *dev_ptr = static_cast<uint8_t*>(base) + offset;
    return FKV_OK;
}

int fkv_ipc_close(void* dev_ptr, int64_t offset) {
    fkv::clear_error();
    FKV_REQUIRE(dev_ptr != nullptr, FKV_ERR_INVALID, "fkv_ipc_close: NULL pointer");
    FKV_CUDA_CHECK(cudaIpcCloseMemHandle(static_cast<uint8_t*>(dev_ptr) - offset));
    return FKV_OK;
}

int fkv_exchange_combine(int32_t P, int32_t rank, int32_t N, int32_t D, const float* local_block,
                         const uint64_t* peer_recv, void* my_recv, int32_t* state, float spike_margin,
                         uint16_t* out, int32_t* flags, int32_t* tokens, void* stream) {
    fkv::clear_error();
    FKV_REQUIRE(P > 0 && rank >= 0 && rank < P && N > 0, FKV_ERR_INVALID,
                "fkv_exchange_combine: P=%d rank=%d N=%d", P, rank, N);
    FKV_REQUIRE(D == 64 || D == 128, FKV_ERR_UNSUPPORTED, "head dim %d unsupported", D);
    FKV_REQUIRE(local_block && peer_recv && my_recv && state && out && flags && tokens,
                FKV_ERR_INVALID, "fkv_exchange_combine: NULL argument");
    FKV_REQUIRE(((uintptr_t)local_block & 15u) == 0 && ((uintptr_t)my_recv & 63u) == 0,
                FKV_ERR_INVALID, "local block must be 16-byte and receive buffer 64-byte aligned");
    int dev = 0, nsm = 0;
    FKV_CUDA_CHECK(cudaGetDevice(&dev));
    FKV_CUDA_CHECK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    // every block waits for the flags that the last block of each rank sets:
    // all N blocks must be resident at once (small blocks, a few per SM)
    FKV_REQUIRE(N <= 4 * nsm, FKV_ERR_UNSUPPORTED, "N=%d rows exceed the co-resident block limit %d",
                N, 4 * nsm);
    const int64_t stride = fkv_exchange_block_stride(N, D);
    cudaStream_t st = (cudaStream_t)stream;
    if (D == 128)
        exchange_combine_kernel<128><<<N, kExThreads, 0, st>>>(P, rank, N, stride, local_block, peer_recv,
                                                             static_cast<uint8_t*>(my_recv), state,
                                                             spike_margin, out, flags, tokens);
    else
        exchange_combine_kernel<64><<<N, kExThreads, 0, st>>>(P, rank, N, stride, local_block, peer_recv,
                                                            static_cast<uint8_t*>(my_recv), state,
                                                            spike_margin, out, flags, tokens);
    FKV_LAUNCH_CHECK();
    return FKV_OK;
}

}  // extern "C"
