// Tier selection + compression kernels (prefill cache -> near / far tiers).
//
// One warp per output row.  Rows [0, Np) of a (b,h) stream are the near tier
// (gathered fp16, zeroed headroom), rows [Np, Np+F) the far tier (encoded),
// with an optional exact fp16 copy of every far row (the promotion archive).
// The work is a single HBM pass: read 4*D bytes per token, write the tier.
//
// Code semantics follow the reference's Python CPU path:
//   fp8 E4M3  src/foveated_kv/mlx_foveated.py:528-566 (bit arithmetic)
//   INT4 V    src/foveated_kv/mlx_foveated.py:569-600 (IEEE fp32, rint)
//   turbo     src/foveated_kv/turbo_quantize.py:25-178 (fp64 accumulation)
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "fkv_common.h"

namespace {

constexpr int kWarpsPerBlock = 8;

// Two fp16 values (low half first) -> two E4M3 codes (low byte first),
// identical to _fp16_to_e4m3 (mlx_foveated.py:528-566: rebias -8, round-half-
// even 10->3 bits with carry, underflow after carry -> signed zero, overflow /
// inf / nan -> sign|0x76).  The hardware conversion (round to nearest even,
// saturating) agrees with that rounding on the normal range; the reference's
// own edges are applied on the fp16 magnitude: below 0x23C0
// (0.96875 * 2^-6, where the reference's rounded exponent is still <= 0) a
// signed zero, from 0x5BC0 (248, whose rounding carries into exponent 15)
// and for inf / NaN the code sign|0x76.  All 65,536 patterns are tested.
__device__ __forceinline__ uint32_t f16x2_to_e4m3x2(uint32_t w) {
    uint16_t hw;
    asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;\n" : "=h"(hw) : "r"(w));
    uint32_t out = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const uint32_t mag = (w >> (16 * j)) & 0x7FFFu;
        const uint32_t sgn = (w >> (16 * j + 8)) & 0x80u;
        uint32_t byte = ((uint32_t)hw >> (8 * j)) & 0xFFu;
        byte = mag < 0x23C0u ? sgn : (mag >= 0x5BC0u ? (sgn | 0x76u) : byte);
        out |= byte << (8 * j);
    }
    return out;
}

__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// Per-lane slice of one D-wide fp16 row: D/32 consecutive halves.
template <int D>
struct RowSlice {
    static constexpr int N = D / 32;  // halves per lane (2 or 4)
    uint16_t h[N];
};

template <int D>
__device__ __forceinline__ void load_row(const uint16_t* __restrict__ src, int lane,
                                         RowSlice<D>& r) {
    if constexpr (D == 128) {
        const uint2 w = __ldg(reinterpret_cast<const uint2*>(src) + lane);
        r.h[0] = w.x & 0xFFFF; r.h[1] = w.x >> 16; r.h[2] = w.y & 0xFFFF; r.h[3] = w.y >> 16;
    } else {
        const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(src) + lane);
        r.h[0] = w & 0xFFFF; r.h[1] = w >> 16;
    }
}

template <int D>
__device__ __forceinline__ void store_row(uint16_t* __restrict__ dst, int lane,
                                          const RowSlice<D>& r) {
    if constexpr (D == 128) {
        uint2 w;
        w.x = (uint32_t)r.h[0] | ((uint32_t)r.h[1] << 16);
        w.y = (uint32_t)r.h[2] | ((uint32_t)r.h[3] << 16);
        reinterpret_cast<uint2*>(dst)[lane] = w;
    } else {
        reinterpret_cast<uint32_t*>(dst)[lane] = (uint32_t)r.h[0] | ((uint32_t)r.h[1] << 16);
    }
}

template <int D>
__device__ __forceinline__ void zero_row(uint16_t* __restrict__ dst, int lane) {
    RowSlice<D> z;
#pragma unroll
    for (int i = 0; i < RowSlice<D>::N; ++i) z.h[i] = 0;
    store_row<D>(dst, lane, z);
}

// min/max over `width` consecutive lanes (width power of two, <= 32)
__device__ __forceinline__ void group_minmax(float& mn, float& mx, int width) {
    for (int o = 1; o < width; o <<= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
}

__global__ void select_recency_kernel(FkvTierLayout L, int streams, int32_t* __restrict__ near_idx,
                                      int32_t* __restrict__ far_idx,
                                      int32_t* __restrict__ near_valid) {
    const int Np = L.n_near_padded, F = L.far_count;
    const int s = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < Np + F; i += gridDim.x * blockDim.x) {
        if (i < Np) {
            int pos = -1;
            if (i < L.n_sinks) pos = i;
            else if (i < L.n_sinks + L.near_from_mid) pos = L.near_mid_start + (i - L.n_sinks);
            else if (i < L.r_actual) pos = L.S - L.window + (i - L.n_sinks - L.near_from_mid);
            near_idx[(int64_t)s * Np + i] = pos;
        } else {
            far_idx[(int64_t)s * F + (i - Np)] = L.mid_start + (i - Np);
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) near_valid[s] = L.r_actual;
    (void)streams;
}

// fp8 K + INT4 V (per-token when VG == 0, else groups of VG dims).
template <int D, int VG>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    compress_fp8_kernel(FkvTierLayout L, const uint16_t* __restrict__ k,
                        const uint16_t* __restrict__ v, int64_t kv_stride_bh,
                        const int32_t* __restrict__ near_idx, const int32_t* __restrict__ far_idx,
                        uint16_t* __restrict__ near_k, uint16_t* __restrict__ near_v,
                        uint8_t* __restrict__ far_k, uint8_t* __restrict__ far_v,
                        uint16_t* __restrict__ v_scale, uint16_t* __restrict__ v_zero,
                        uint16_t* __restrict__ arc_k, uint16_t* __restrict__ arc_v) {
    constexpr int N = D / 32;
    const int Np = L.n_near_padded, F = L.far_count;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
    const int64_t s = blockIdx.y;
    if (row >= Np + F) return;
    const uint16_t* ks = k + s * kv_stride_bh;
    const uint16_t* vs = v + s * kv_stride_bh;
    if (row < Np) {
        const int pos = near_idx[s * Np + row];
        uint16_t* dk = near_k + (s * Np + row) * D;
        uint16_t* dv = near_v + (s * Np + row) * D;
        if (pos < 0) {
            zero_row<D>(dk, lane);
            zero_row<D>(dv, lane);
        } else {
            RowSlice<D> a, b;
            load_row<D>(ks + (int64_t)pos * D, lane, a);
            load_row<D>(vs + (int64_t)pos * D, lane, b);
            store_row<D>(dk, lane, a);
            store_row<D>(dv, lane, b);
        }
        return;
    }
    const int f = row - Np;
    const int64_t frow = s * F + f;
    const int pos = far_idx[frow];
    RowSlice<D> a, b;
    load_row<D>(ks + (int64_t)pos * D, lane, a);
    load_row<D>(vs + (int64_t)pos * D, lane, b);
    if (arc_k != nullptr) store_row<D>(arc_k + frow * D, lane, a);
    if (arc_v != nullptr) store_row<D>(arc_v + frow * D, lane, b);

    // K: E4M3 codes, lane owns dims [lane*N, lane*N+N)
    uint32_t kc = 0;
#pragma unroll
    for (int i = 0; i < N; i += 2)
        kc |= f16x2_to_e4m3x2((uint32_t)a.h[i] | ((uint32_t)a.h[i + 1] << 16)) << (8 * i);
    if constexpr (N == 4) reinterpret_cast<uint32_t*>(far_k + frow * D)[lane] = kc;
    else reinterpret_cast<uint16_t*>(far_k + frow * D)[lane] = (uint16_t)kc;

    // V: asymmetric INT4 over the token (or group), fp32 as the reference.
    float x[N];
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        x[i] = h2f(b.h[i]);
        mn = fminf(mn, x[i]);
        mx = fmaxf(mx, x[i]);
    }
    constexpr int width = (VG == 0) ? 32 : VG / N;  // lanes per quantisation group
    group_minmax(mn, mx, width);
    float scale = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    if (scale == 0.0f) scale = 1.0f;
    // code = rint((x - mn) / scale) with the IEEE fp32 quotient.  The
    // quotient lies in [0, ~15]; the product with the rounded reciprocal is
    // within ~2e-6 of it, so rint agrees unless the product sits within 1e-4
    // of a rounding boundary (k + 0.5) -- only then (or for non-finite
    // values) is the correctly rounded division evaluated.
    const float rcp = __frcp_rn(scale);
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const float d = __fsub_rn(x[i], mn);
        float qa = __fmul_rn(d, rcp);
        const float fr = qa - floorf(qa);
        if (!(fabsf(fr - 0.5f) > 1e-4f)) qa = __fdiv_rn(d, scale);
        float q = rintf(qa);
        q = fminf(fmaxf(q, 0.0f), 15.0f);
        packed |= ((uint32_t)q) << (4 * i);
    }
    // N dims -> N/2 bytes per lane, even dim in the low nibble
    if constexpr (N == 4) reinterpret_cast<uint16_t*>(far_v + frow * (D / 2))[lane] = (uint16_t)packed;
    else far_v[frow * (D / 2) + lane] = (uint8_t)packed;
    if constexpr (VG == 0) {
        if (lane == 0) {
            v_scale[frow] = __half_as_ushort(__float2half_rn(scale));
            v_zero[frow] = __half_as_ushort(__float2half_rn(mn));
        }
    } else {
        if ((lane % width) == 0) {
            const int g = lane / width;
            v_scale[frow * (D / VG) + g] = __half_as_ushort(__float2half_rn(scale));
            v_zero[frow * (D / VG) + g] = __half_as_ushort(__float2half_rn(mn));
        }
    }
}

// TurboQuant far tier.  Pi and S are staged once per block in shared memory
// (rows padded to D+1 floats so a warp reading one column is conflict-free);
// each warp then encodes far tokens in fp64.
template <int D>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    compress_turbo_kernel(FkvTierLayout L, int streams, const uint16_t* __restrict__ k,
                          const uint16_t* __restrict__ v, int64_t kv_stride_bh,
                          const int32_t* __restrict__ near_idx,
                          const int32_t* __restrict__ far_idx, const float* __restrict__ Pi,
                          const float* __restrict__ Smat, const float* __restrict__ centroids,
                          const float* __restrict__ boundaries, uint16_t* __restrict__ near_k,
                          uint16_t* __restrict__ near_v, uint8_t* __restrict__ k_idx,
                          uint8_t* __restrict__ k_signs, uint16_t* __restrict__ k_norm,
                          uint16_t* __restrict__ k_gamma, uint8_t* __restrict__ v_packed,
                          uint16_t* __restrict__ v_scale, uint16_t* __restrict__ arc_k,
                          uint16_t* __restrict__ arc_v) {
    constexpr int P = D + 1;     // padded row stride
    constexpr int U = D / 32;    // outputs per lane
    extern __shared__ float smem[];
    float* sPi = smem;           // [D][P]
    float* sS = smem + D * P;    // [D][P]
    double* svec = reinterpret_cast<double*>(sS + D * P);   // [warps][D]
    uint8_t* scode = reinterpret_cast<uint8_t*>(svec + kWarpsPerBlock * D);  // [warps][D]
    for (int i = threadIdx.x; i < D * D; i += blockDim.x) {
        sPi[(i / D) * P + (i % D)] = Pi[i];
        sS[(i / D) * P + (i % D)] = Smat[i];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    double* vec = svec + w * D;
    uint8_t* code = scode + w * D;
    const int Np = L.n_near_padded, F = L.far_count;
    const int64_t total = (int64_t)streams * (Np + F);
    const double c0 = centroids[0], c1 = centroids[1], c2 = centroids[2], c3 = centroids[3];
    const double b0 = boundaries[0], b1 = boundaries[1], b2 = boundaries[2];
    for (int64_t item = (int64_t)blockIdx.x * kWarpsPerBlock + w; item < total;
         item += (int64_t)gridDim.x * kWarpsPerBlock) {
        const int64_t s = item / (Np + F);
        const int row = (int)(item % (Np + F));
        const uint16_t* ks = k + s * kv_stride_bh;
        const uint16_t* vs = v + s * kv_stride_bh;
        if (row < Np) {
            const int pos = near_idx[s * Np + row];
            uint16_t* dk = near_k + (s * Np + row) * D;
            uint16_t* dv = near_v + (s * Np + row) * D;
            if (pos < 0) {
                zero_row<D>(dk, lane);
                zero_row<D>(dv, lane);
            } else {
                RowSlice<D> a, b;
                load_row<D>(ks + (int64_t)pos * D, lane, a);
                load_row<D>(vs + (int64_t)pos * D, lane, b);
                store_row<D>(dk, lane, a);
                store_row<D>(dv, lane, b);
            }
            continue;
        }
        const int64_t frow = s * F + (row - Np);
        const int pos = far_idx[frow];
        RowSlice<D> a, b;
        load_row<D>(ks + (int64_t)pos * D, lane, a);
        load_row<D>(vs + (int64_t)pos * D, lane, b);
        if (arc_k != nullptr) store_row<D>(arc_k + frow * D, lane, a);
        if (arc_v != nullptr) store_row<D>(arc_v + frow * D, lane, b);

        // ---- K: norm, rotate, 2-bit Lloyd-Max, residual, QJL signs (fp64)
        double kx[U];
        double ss = 0.0;
#pragma unroll
        for (int i = 0; i < U; ++i) {
            kx[i] = (double)h2f(a.h[i]);
            ss += kx[i] * kx[i];
        }
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const double nrm = sqrt(ss);
        const double inv = 1.0 / fmax(nrm, 1e-8);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < U; ++i) vec[lane * U + i] = kx[i] * inv;
        __syncwarp();
        // y_j = sum_i kn_i Pi[j][i]  for j = lane + 32u
        int idxv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = lane + 32 * u;
            double y = 0.0;
            for (int i = 0; i < D; ++i) y = fma(vec[i], (double)sPi[j * P + i], y);
            idxv[u] = (y >= b0) + (y >= b1) + (y >= b2);
            code[j] = (uint8_t)idxv[u];
        }
        __syncwarp();
        // k_hat_i = nrm * sum_j c[idx_j] Pi[j][i] ; residual r_i = k_i - k_hat_i
        double cv_local[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int id = idxv[u];
            cv_local[u] = id == 0 ? c0 : (id == 1 ? c1 : (id == 2 ? c2 : c3));
        }
        __syncwarp();
#pragma unroll
        for (int u = 0; u < U; ++u) vec[lane + 32 * u] = cv_local[u];
        __syncwarp();
        double r[U];
        double gs = 0.0;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = lane * U + u;   // dims owned as in kx[]
            double acc = 0.0;
            for (int j = 0; j < D; ++j) acc = fma(vec[j], (double)sPi[j * P + i], acc);
            r[u] = kx[u] - nrm * acc;
            gs += r[u] * r[u];
        }
        for (int o = 16; o > 0; o >>= 1) gs += __shfl_xor_sync(0xffffffffu, gs, o);
        __syncwarp();
#pragma unroll
        for (int u = 0; u < U; ++u) vec[lane * U + u] = r[u];
        __syncwarp();
        // proj_j = sum_i r_i S[j][i] ; sign bit = proj >= 0
        uint8_t sbits[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = lane + 32 * u;
            double pj = 0.0;
            for (int i = 0; i < D; ++i) pj = fma(vec[i], (double)sS[j * P + i], pj);
            sbits[u] = pj >= 0.0 ? 1 : 0;
        }
        __syncwarp();
        // pack: 2-bit codes (dim 4m+i -> bits 2i), then signs (dim 8m+i -> bit i)
        if (lane < D / 4) {
            const uint8_t* cc = code + 4 * lane;
            k_idx[frow * (D / 4) + lane] =
                (uint8_t)(cc[0] | (cc[1] << 2) | (cc[2] << 4) | (cc[3] << 6));
        }
        __syncwarp();
#pragma unroll
        for (int u = 0; u < U; ++u) code[lane + 32 * u] = sbits[u];
        __syncwarp();
        if (lane < D / 8) {
            const uint8_t* cc = code + 8 * lane;
            uint32_t byte = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) byte |= (uint32_t)cc[i] << i;
            k_signs[frow * (D / 8) + lane] = (uint8_t)byte;
        }
        if (lane == 0) {
            k_norm[frow] = __half_as_ushort(__double2half(nrm));
            k_gamma[frow] = __half_as_ushort(__double2half(sqrt(gs)));
        }
        __syncwarp();

        // ---- V: 2-bit symmetric, groups of 32 dims (fp32 as the reference)
        float x[U];
        float am = 0.0f;
#pragma unroll
        for (int i = 0; i < U; ++i) {
            x[i] = h2f(b.h[i]);
            am = fmaxf(am, fabsf(x[i]));
        }
        constexpr int width = 32 / U;   // lanes per 32-dim group
        for (int o = 1; o < width; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        const float sc = fmaxf(am, 1e-8f);
        uint32_t q4 = 0;
#pragma unroll
        for (int i = 0; i < U; ++i) {
            float t = rintf(__fmul_rn(__fadd_rn(__fdiv_rn(x[i], sc), 1.0f), 1.5f));
            t = fminf(fmaxf(t, 0.0f), 3.0f);
            q4 |= ((uint32_t)t) << (2 * i);
        }
        if constexpr (U == 4) {
            v_packed[frow * (D / 4) + lane] = (uint8_t)q4;
        } else {   // U == 2: two lanes form one byte
            const uint32_t other = __shfl_down_sync(0xffffffffu, q4, 1);
            if ((lane & 1) == 0) v_packed[frow * (D / 4) + lane / 2] = (uint8_t)(q4 | (other << 4));
        }
        if ((lane % width) == 0) v_scale[frow * (D / 32) + lane / width] =
            __half_as_ushort(__float2half_rn(sc));
    }
}

int check_common(const FkvTierLayout* L, int B, int Hk, int D, const void* k, const void* v,
                 int64_t stride) {
    FKV_REQUIRE(L != nullptr, FKV_ERR_INVALID, "tier layout is NULL");
    FKV_REQUIRE(B > 0 && Hk > 0, FKV_ERR_INVALID, "B=%d Hk=%d must be positive", B, Hk);
    FKV_REQUIRE(D == 64 || D == 128, FKV_ERR_UNSUPPORTED, "head dim %d unsupported (64, 128)", D);
    FKV_REQUIRE(k != nullptr && v != nullptr, FKV_ERR_INVALID, "k/v pointer is NULL");
    FKV_REQUIRE(stride >= (int64_t)L->S * D, FKV_ERR_INVALID,
                "kv_stride_bh=%lld smaller than S*D=%lld", (long long)stride,
                (long long)L->S * D);
    FKV_REQUIRE(((uintptr_t)k % 16) == 0 && ((uintptr_t)v % 16) == 0, FKV_ERR_INVALID,
                "k/v must be 16-byte aligned");
    return FKV_OK;
}

}  // namespace

extern "C" {

int fkv_select_recency(const FkvTierLayout* L, int32_t B, int32_t Hk, int32_t* near_idx,
                       int32_t* far_idx, int32_t* near_valid, void* stream) {
    fkv::clear_error();
    FKV_REQUIRE(L != nullptr && near_idx && near_valid && (far_idx || L->far_count == 0),
                FKV_ERR_INVALID, "fkv_select_recency: NULL argument");
    FKV_REQUIRE(B > 0 && Hk > 0, FKV_ERR_INVALID, "B=%d Hk=%d must be positive", B, Hk);
    const int total = L->n_near_padded + L->far_count;
    dim3 grid((total + 255) / 256, B * Hk);
    select_recency_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(*L, B * Hk, near_idx, far_idx,
                                                                   near_valid);
    FKV_LAUNCH_CHECK();
    return FKV_OK;
}

int fkv_compress_fp8(const FkvTierLayout* L, int32_t B, int32_t Hk, int32_t D,
                     const uint16_t* k, const uint16_t* v, int64_t kv_stride_bh,
                     const int32_t* near_idx, const int32_t* far_idx, int32_t v_group,
                     uint16_t* near_k, uint16_t* near_v, uint8_t* far_k, uint8_t* far_v,
                     uint16_t* v_scale, uint16_t* v_zero, uint16_t* arc_k, uint16_t* arc_v,
                     void* stream) {
    fkv::clear_error();
    int rc = check_common(L, B, Hk, D, k, v, kv_stride_bh);
    if (rc) return rc;
    FKV_REQUIRE(v_group == 0 || v_group == 32, FKV_ERR_UNSUPPORTED,
                "v_group=%d unsupported (0 = per token, 32)", v_group);
    FKV_REQUIRE(near_idx && near_k && near_v, FKV_ERR_INVALID, "near pointers are NULL");
    FKV_REQUIRE(L->far_count == 0 || (far_idx && far_k && far_v && v_scale && v_zero),
                FKV_ERR_INVALID, "far pointers are NULL");
    const int rows = L->n_near_padded + L->far_count;
    if (rows == 0) return FKV_OK;
    dim3 grid((rows + kWarpsPerBlock - 1) / kWarpsPerBlock, B * Hk);
    auto st = (cudaStream_t)stream;
#define FKV_LAUNCH(DD, VV)                                                                    \
    compress_fp8_kernel<DD, VV><<<grid, kWarpsPerBlock * 32, 0, st>>>(                        \
        *L, k, v, kv_stride_bh, near_idx, far_idx, near_k, near_v, far_k, far_v, v_scale,     \
        v_zero, arc_k, arc_v)
    if (D == 128) {
        if (v_group == 0) FKV_LAUNCH(128, 0); else FKV_LAUNCH(128, 32);
    } else {
        if (v_group == 0) FKV_LAUNCH(64, 0); else FKV_LAUNCH(64, 32);
    }
#undef FKV_LAUNCH
    FKV_LAUNCH_CHECK();
    return FKV_OK;
}

int fkv_compress_turbo(const FkvTierLayout* L, int32_t B, int32_t Hk, int32_t D,
                       const uint16_t* k, const uint16_t* v, int64_t kv_stride_bh,
                       const int32_t* near_idx, const int32_t* far_idx,
                       const float* Pi, const float* Smat, const float* centroids,
                       const float* boundaries, uint16_t* near_k, uint16_t* near_v,
                       uint8_t* k_idx, uint8_t* k_signs, uint16_t* k_norm, uint16_t* k_gamma,
                       uint8_t* v_packed, uint16_t* v_scale, uint16_t* arc_k, uint16_t* arc_v,
                       void* stream) {
    fkv::clear_error();
    int rc = check_common(L, B, Hk, D, k, v, kv_stride_bh);
    if (rc) return rc;
    FKV_REQUIRE(Pi && Smat && centroids && boundaries, FKV_ERR_INVALID,
                "turbo constants are NULL");
    FKV_REQUIRE(near_idx && near_k && near_v, FKV_ERR_INVALID, "near pointers are NULL");
    FKV_REQUIRE(L->far_count == 0 || (far_idx && k_idx && k_signs && k_norm && k_gamma &&
                                      v_packed && v_scale),
                FKV_ERR_INVALID, "far pointers are NULL");
    const int64_t rows = (int64_t)B * Hk * (L->n_near_padded + L->far_count);
    if (rows == 0) return FKV_OK;
    const size_t smem = (size_t)2 * D * (D + 1) * sizeof(float) +
                        (size_t)kWarpsPerBlock * D * (sizeof(double) + 1);
    auto st = (cudaStream_t)stream;
    int dev = 0, nsm = 148;
    FKV_CUDA_CHECK(cudaGetDevice(&dev));
    FKV_CUDA_CHECK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    const int64_t want = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
    const int grid = (int)(want < (int64_t)nsm ? want : (int64_t)nsm);
    if (D == 128) {
        FKV_CUDA_CHECK(cudaFuncSetAttribute(compress_turbo_kernel<128>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem));
        compress_turbo_kernel<128><<<grid, kWarpsPerBlock * 32, smem, st>>>(
            *L, B * Hk, k, v, kv_stride_bh, near_idx, far_idx, Pi, Smat, centroids, boundaries,
            near_k, near_v, k_idx, k_signs, k_norm, k_gamma, v_packed, v_scale, arc_k, arc_v);
    } else {
        FKV_CUDA_CHECK(cudaFuncSetAttribute(compress_turbo_kernel<64>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem));
        compress_turbo_kernel<64><<<grid, kWarpsPerBlock * 32, smem, st>>>(
            *L, B * Hk, k, v, kv_stride_bh, near_idx, far_idx, Pi, Smat, centroids, boundaries,
            near_k, near_v, k_idx, k_signs, k_norm, k_gamma, v_packed, v_scale, arc_k, arc_v);
    }
    FKV_LAUNCH_CHECK();
    return FKV_OK;
}

}  // extern "C"
