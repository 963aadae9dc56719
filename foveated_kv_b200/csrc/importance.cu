// Importance-ranked tier selection (the reference selects by recency only;
// this follows the specification its README and paper describe).
//
// Per (b, kv head) stream with G query heads q_obs:
//   s_g[t]  = q_g . k_t / sqrt(D)                         (fp64)
//   imp[t]  = sum_g exp(s_g[t] - max_t s_g) / sum_t exp(s_g[t] - max_t s_g)
// Sinks and the recency window are always near; the near_from_mid middle
// tokens with the largest imp (ties to the lower position) join them.  Near
// order: sinks, selected middle ascending, window; far: the rest of the
// middle ascending.  Four launches: scores, per-head softmax statistics,
// importance, and one block per stream doing a radix select of the k-th
// largest importance followed by an ordered compaction.
#include <cub/block/block_scan.cuh>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "fkv_common.h"

namespace {

constexpr int kSelThreads = 1024;

// scores[s][g][t], one warp per token
__global__ void imp_scores_kernel(FkvTierLayout L, int Hk, int Hq, int D,
                                  const uint16_t* __restrict__ k, int64_t stride,
                                  const uint16_t* __restrict__ q, double* __restrict__ scores) {
    extern __shared__ double qs[];   // [G][D]
    const int G = Hq / Hk;
    const int s = blockIdx.y;
    const int b = s / Hk, h = s % Hk;
    for (int i = threadIdx.x; i < G * D; i += blockDim.x)
        qs[i] = (double)__half2float(__ushort_as_half(q[((int64_t)b * Hq + h * G) * D + i]));
    __syncthreads();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const double inv = 1.0 / sqrt((double)D);
    const uint16_t* ks = k + (int64_t)s * stride;
    for (int t = blockIdx.x * nw + w; t < L.S; t += gridDim.x * nw) {
        double kv[4];
        const int per = D / 32;
        for (int i = 0; i < per; ++i)
            kv[i] = (double)__half2float(__ushort_as_half(ks[(int64_t)t * D + lane * per + i]));
        for (int g = 0; g < G; ++g) {
            double a = 0.0;
            for (int i = 0; i < per; ++i) a = fma(qs[g * D + lane * per + i], kv[i], a);
            for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            if (lane == 0) scores[((int64_t)s * G + g) * L.S + t] = a * inv;
        }
    }
}

// stats[s][g] = (max, sum exp(s - max))
__global__ void imp_stats_kernel(int S, const double* __restrict__ scores, double* __restrict__ stats) {
    __shared__ double red[32];
    const int row = blockIdx.x;   // s * G + g
    const double* x = scores + (int64_t)row * S;
    double m = -INFINITY;
    for (int t = threadIdx.x; t < S; t += blockDim.x) m = fmax(m, x[t]);
    for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
        for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (threadIdx.x == 0) red[0] = m;
    }
    __syncthreads();
    m = red[0];
    __syncthreads();
    double z = 0.0;
    for (int t = threadIdx.x; t < S; t += blockDim.x) z += exp(x[t] - m);
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = z;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
        stats[2 * row] = m;
        stats[2 * row + 1] = tot;
    }
}

// imp[s][t] (as IEEE bits: non-negative doubles order like unsigned integers)
__global__ void imp_combine_kernel(int S, int G, const double* __restrict__ scores,
                                   const double* __restrict__ stats, uint64_t* __restrict__ imp) {
    const int s = blockIdx.y;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < S; t += gridDim.x * blockDim.x) {
        double v = 0.0;
        for (int g = 0; g < G; ++g) {
            const int row = s * G + g;
            v += exp(scores[(int64_t)row * S + t] - stats[2 * row]) / stats[2 * row + 1];
        }
        imp[(int64_t)s * S + t] = (uint64_t)__double_as_longlong(v);
    }
}

__global__ void __launch_bounds__(kSelThreads)
    imp_select_kernel(FkvTierLayout L, const uint64_t* __restrict__ imp,
                      int32_t* __restrict__ near_idx, int32_t* __restrict__ far_idx,
                      int32_t* __restrict__ near_valid) {
    using Scan = cub::BlockScan<int, kSelThreads>;
    __shared__ typename Scan::TempStorage scan_tmp;
    __shared__ unsigned int hist[256];
    __shared__ uint64_t sh_prefix;
    __shared__ int sh_krem;
    __shared__ int sh_run[3];
    const int s = blockIdx.x, tid = threadIdx.x;
    const int Np = L.n_near_padded, F = L.far_count;
    const int ms = L.mid_start, me = L.mid_end, k = L.near_from_mid;
    const uint64_t* x = imp + (int64_t)s * L.S;
    int32_t* ni = near_idx + (int64_t)s * Np;
    int32_t* fi = far_idx + (int64_t)s * F;

    // ---- radix select: T = k-th largest key among the middle tokens
    uint64_t prefix = 0;
    int krem = k;
    if (k > 0) {
        for (int pass = 7; pass >= 0; --pass) {
            const int shift = 8 * pass;
            const uint64_t hmask = pass == 7 ? 0ull : (~0ull << (shift + 8));
            for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
            __syncthreads();
            for (int t = ms + tid; t < me; t += kSelThreads) {
                const uint64_t v = x[t];
                if ((v & hmask) == (prefix & hmask)) atomicAdd(&hist[(v >> shift) & 0xFF], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                int acc = 0, d = 255;
                for (; d > 0; --d) {
                    if (acc + (int)hist[d] >= krem) break;
                    acc += hist[d];
                }
                sh_krem = krem - acc;
                sh_prefix = prefix | ((uint64_t)d << shift);
            }
            __syncthreads();
            prefix = sh_prefix;
            krem = sh_krem;
            __syncthreads();
        }
    }
    // selected: key > T, or key == T among the first `krem` equal keys by position
    if (tid == 0) {
        sh_run[0] = 0;   // equal keys seen
        sh_run[1] = 0;   // selected so far
        sh_run[2] = 0;   // unselected so far
    }
    __syncthreads();
    for (int base = ms; base < me; base += kSelThreads) {
        const int t = base + tid;
        const bool in = t < me;
        const uint64_t v = in ? x[t] : 0ull;
        const bool eq = in && k > 0 && v == prefix;
        int eq_before, eq_tot;
        Scan(scan_tmp).ExclusiveSum(eq ? 1 : 0, eq_before, eq_tot);
        __syncthreads();
        const bool sel = in && k > 0 && (v > prefix || (eq && sh_run[0] + eq_before < krem));
        const bool uns = in && !sel;
        int sel_before, sel_tot, uns_before, uns_tot;
        Scan(scan_tmp).ExclusiveSum(sel ? 1 : 0, sel_before, sel_tot);
        __syncthreads();
        Scan(scan_tmp).ExclusiveSum(uns ? 1 : 0, uns_before, uns_tot);
        if (sel) ni[L.n_sinks + sh_run[1] + sel_before] = t;
        if (uns) fi[sh_run[2] + uns_before] = t;
        __syncthreads();
        if (tid == 0) {
            sh_run[0] += eq_tot;
            sh_run[1] += sel_tot;
            sh_run[2] += uns_tot;
        }
        __syncthreads();
    }
    for (int i = tid; i < Np; i += kSelThreads) {
        if (i < L.n_sinks) ni[i] = i;
        else if (i >= L.n_sinks + L.near_from_mid && i < L.r_actual)
            ni[i] = L.S - L.window + (i - L.n_sinks - L.near_from_mid);
        else if (i >= L.r_actual) ni[i] = -1;
    }
    if (tid == 0) near_valid[s] = L.r_actual;
}

struct ImpLayout {
    size_t scores, stats, imp, total;
};

ImpLayout imp_layout(const FkvTierLayout* L, int B, int Hk, int Hq) {
    const size_t streams = (size_t)B * Hk, G = (size_t)(Hq / Hk);
    ImpLayout o;
    o.scores = 0;
    o.stats = o.scores + ((streams * G * L->S * sizeof(double) + 255) & ~(size_t)255);
    o.imp = o.stats + ((streams * G * 2 * sizeof(double) + 255) & ~(size_t)255);
    o.total = o.imp + streams * L->S * sizeof(uint64_t) + 256;
    return o;
}

}  // namespace

extern "C" {

size_t fkv_select_importance_workspace_bytes(const FkvTierLayout* L, int32_t B, int32_t Hk,
                                             int32_t Hq) {
    if (!L || B <= 0 || Hk <= 0 || Hq <= 0 || Hq % Hk) return 0;
    return imp_layout(L, B, Hk, Hq).total;
}

int fkv_select_importance(const FkvTierLayout* L, int32_t B, int32_t Hk, int32_t Hq, int32_t D,
                          const uint16_t* k, int64_t kv_stride_bh, const uint16_t* q_obs,
                          int32_t* near_idx, int32_t* far_idx, int32_t* near_valid,
                          void* workspace, size_t workspace_bytes, void* stream) {
    fkv::clear_error();
    FKV_REQUIRE(L && k && q_obs && near_idx && near_valid && (far_idx || L->far_count == 0),
                FKV_ERR_INVALID, "fkv_select_importance: NULL argument");
    FKV_REQUIRE(B > 0 && Hk > 0 && Hq > 0 && Hq % Hk == 0, FKV_ERR_INVALID,
                "B=%d Hk=%d Hq=%d invalid", B, Hk, Hq);
    FKV_REQUIRE(D == 64 || D == 128, FKV_ERR_UNSUPPORTED, "head dim %d unsupported", D);
    FKV_REQUIRE(kv_stride_bh >= (int64_t)L->S * D, FKV_ERR_INVALID, "kv_stride_bh too small");
    FKV_REQUIRE(Hq / Hk <= 64, FKV_ERR_UNSUPPORTED, "GQA group %d > 64", Hq / Hk);
    const ImpLayout lay = imp_layout(L, B, Hk, Hq);
    FKV_REQUIRE(workspace && workspace_bytes >= lay.total, FKV_ERR_INVALID,
                "workspace too small: %zu < %zu bytes", workspace_bytes, lay.total);
    const int streams = B * Hk, G = Hq / Hk;
    auto st = (cudaStream_t)stream;
    char* ws = static_cast<char*>(workspace);
    double* scores = reinterpret_cast<double*>(ws + lay.scores);
    double* stats = reinterpret_cast<double*>(ws + lay.stats);
    uint64_t* imp = reinterpret_cast<uint64_t*>(ws + lay.imp);
    if (L->S > 0) {
        const size_t qsm = (size_t)G * D * sizeof(double);
        if (qsm > 48 * 1024)
            FKV_CUDA_CHECK(cudaFuncSetAttribute(imp_scores_kernel,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)qsm));
        dim3 g1((L->S + 63) / 64, streams);
        imp_scores_kernel<<<g1, 256, qsm, st>>>(*L, Hk, Hq, D, k, kv_stride_bh, q_obs, scores);
        FKV_LAUNCH_CHECK();
        imp_stats_kernel<<<streams * G, 512, 0, st>>>(L->S, scores, stats);
        FKV_LAUNCH_CHECK();
        dim3 g3((L->S + 255) / 256, streams);
        imp_combine_kernel<<<g3, 256, 0, st>>>(L->S, G, scores, stats, imp);
        FKV_LAUNCH_CHECK();
    }
    imp_select_kernel<<<streams, kSelThreads, 0, st>>>(*L, imp, near_idx, far_idx, near_valid);
    FKV_LAUNCH_CHECK();
    return FKV_OK;
}

}  // extern "C"
