// Sequence-split exchange over NVLink peer memory, fused with the merge.
//
// Each rank of a sequence split holds one block of partial records
// ([N records of (m, l, min_near, max_far, o[D])] followed by N argmax
// values) after its partial decode.  fkv_exchange_combine replaces the
// all-gather + merge of that step with ONE kernel launch per rank.  Block n
// handles output row n:
//
//   1. it sends row n of the local block (D + 4 record words and the argmax)
//      to slot `rank` of every rank's receive buffer, each 4-byte word paired
//      with the step's sequence number in one 8-byte store (plain stores to
//      the peers' memory through CUDA IPC mappings over NVLink; no TMA, no
//      multicast).  A word and its tag land together, so no fence or flag is
//      needed (the low-latency protocol NCCL calls LL);
//   2. it polls (bounded) its own receive buffer until row n of all P ranks
//      carries the step's tag, staging the values in shared memory;
//   3. it merges the P records in rank order (earliest rank wins max_far
//      ties), as fkv_combine_partials does.
//
// Receive buffers are double-buffered by the parity of the sequence number:
// a rank can only write step t + 2 into a peer after its own step t + 1
// merge, which needed the peer's step t + 1 rows, which the peer sent after
// finishing its step t merge -- so no slot is overwritten while it is read,
// and a stale word (tag t) never passes for a fresh one (tag t + 2).  The
// sequence number lives in device memory (state[0]) and is advanced by the
// launch itself, so a captured step replays correctly.
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
constexpr int kExMaxRanks = 8;
constexpr uint32_t kExSpinLimit = 1u << 22;   // polls of one word, ~0.1 us each: under a second

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// words per row: D + 4 record floats and the argmax
__host__ __device__ constexpr int ex_row_words(int D) { return D + 5; }

// Receive buffer of one rank: [2 parities][P ranks][N rows][D + 5] tagged
// 8-byte words (low half: the value's bits, high half: the sequence number).
template <int D>
__global__ void __launch_bounds__(kExThreads)
    exchange_combine_kernel(int P, int rank, int N, int64_t stride, const float* __restrict__ local,
                            const uint64_t* __restrict__ peers, uint64_t* __restrict__ mine,
                            int32_t* __restrict__ state, float margin, uint16_t* __restrict__ out,
                            int32_t* __restrict__ flags, int32_t* __restrict__ tokens) {
    constexpr int RW = ex_row_words(D);
    const int n = blockIdx.x, tid = threadIdx.x;
    __shared__ int sh_seq;
    __shared__ float rec[kExMaxRanks][RW];
    if (tid == 0) sh_seq = *reinterpret_cast<volatile int32_t*>(state) + 1;
    __syncthreads();
    const int seq = sh_seq, par = seq & 1;
    const uint64_t tag = (uint64_t)(uint32_t)seq << 32;
    const float* lrow = local + (int64_t)n * (D + 4);
    const int32_t larg = reinterpret_cast<const int32_t*>(local + (int64_t)N * (D + 4))[n];
    // 1. send row n to every rank
    for (int w = tid; w < RW; w += kExThreads) {
        const uint32_t bits = w < D + 4 ? __float_as_uint(lrow[w]) : (uint32_t)larg;
        const uint64_t word = tag | bits;
        for (int r = 0; r < P; ++r) {
            uint64_t* dst = reinterpret_cast<uint64_t*>(peers[r]) +
                            (((int64_t)par * P + rank) * N + n) * RW + w;
            st_relaxed_sys_u64(dst, word);
        }
    }
    // 2. receive row n of every rank (bounded polls)
    for (int w = tid; w < RW; w += kExThreads) {
        // one round of loads for all ranks first, then re-poll the words
        // that have not arrived yet
        uint64_t v[kExMaxRanks];
#pragma unroll
        for (int k = 0; k < kExMaxRanks; ++k)
            if (k < P) v[k] = ld_relaxed_sys_u64(mine + (((int64_t)par * P + k) * N + n) * RW + w);
#pragma unroll
        for (int k = 0; k < kExMaxRanks; ++k) {
            if (k >= P) continue;
            const uint64_t* src = mine + (((int64_t)par * P + k) * N + n) * RW + w;
            uint32_t i = 0;
            while ((uint32_t)(v[k] >> 32) != (uint32_t)seq) {
                if (++i > kExSpinLimit) {
                    atomicExch(state + 3, FKV_ERR_TIMEOUT);
                    break;
                }
                __nanosleep(32);
                v[k] = ld_relaxed_sys_u64(src);
            }
            rec[k][w] = __uint_as_float((uint32_t)v[k]);
        }
    }
    __syncthreads();
    // 3. merge the P records of row n in rank order
    float M = -INFINITY;
    for (int k = 0; k < P; ++k) M = fmaxf(M, rec[k][0]);
    for (int d = tid; d < D; d += kExThreads) {
        float L = 0.f, acc = 0.f;
        if (M != -INFINITY) {
            for (int k = 0; k < P; ++k) {
                if (rec[k][0] == -INFINITY) continue;
                const float wgt = exp2f((rec[k][0] - M) * kLog2e);
                L = fmaf(wgt, rec[k][1], L);
                acc = fmaf(wgt, rec[k][4 + d], acc);
            }
        }
        out[(int64_t)n * D + d] = __half_as_ushort(__float2half_rn(L > 0.f ? acc / L : 0.f));
    }
    if (tid == 0) {
        float mn = INFINITY, mf = -INFINITY;
        int af = -1;
        for (int k = 0; k < P; ++k) {
            mn = fminf(mn, rec[k][2]);
            if (rec[k][3] > mf) {   // rank order: the first rank with the strict max wins
                mf = rec[k][3];
                af = __float_as_int(rec[k][D + 4]);
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
    return (size_t)2 * P * N * ex_row_words(D) * sizeof(uint64_t);
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
    FKV_REQUIRE(P > 0 && P <= kExMaxRanks && rank >= 0 && rank < P && N > 0, FKV_ERR_INVALID,
                "fkv_exchange_combine: P=%d (at most %d) rank=%d N=%d", P, kExMaxRanks, rank, N);
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
                                                             static_cast<uint64_t*>(my_recv), state,
                                                             spike_margin, out, flags, tokens);
    else
        exchange_combine_kernel<64><<<N, kExThreads, 0, st>>>(P, rank, N, stride, local_block, peer_recv,
                                                            static_cast<uint64_t*>(my_recv), state,
                                                            spike_margin, out, flags, tokens);
    FKV_LAUNCH_CHECK();
    return FKV_OK;
}

}  // extern "C"
