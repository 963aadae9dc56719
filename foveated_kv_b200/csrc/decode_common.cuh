// Device building blocks shared by the fused decode kernels.
//
// Tile = 16 tokens of one (b, kv-head) stream, processed by one warp with two
// m16n8k16 tensor-core products:
//
//   S  (16 x 16 tok)  = Q (16 x D) . K^T   rows 0..7: q_hi of up to 8 q heads
//                                          rows 8..15: q_lo (q - q_hi) of the same
//   O^T (D x 8 heads) += V^T (D x 16 tok) . P^T (16 tok x 8 heads)
//
// Register layout per lane (r = lane/4, c = lane%4):
//   * the QK B fragment of token n (= r) is 4 consecutive bytes of that
//     token's row chunk [c*D/4, (c+1)*D/4): the K dimension is permuted, and
//     Q uses the same permutation, so every lane loads contiguous bytes;
//   * S C-fragments give lane (r, c) the scores of head r for tokens
//     2c, 2c+1, 8+2c, 9+2c -- exactly the P^T B fragment of the PV product;
//   * the V^T A fragment of lane r covers dims [r*D/8, (r+1)*D/8) (output
//     rows permuted: m-tile i, row r -> dim r*D/8 + 2i, row r+8 -> +1).
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace fkvdev {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kHeadsPerTile = 8;

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// two E4M3 codes (low byte -> low half) -> f16x2, exact for every code the
// encoder emits (no subnormal / NaN codes)
__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint32_t two_bytes) {
    __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(two_bytes & 0xFFFFu),
                                                __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

// four E4M3 codes of one word -> (bytes 0,1) and (bytes 2,3) as f16x2 pairs
__device__ __forceinline__ void e4m3x4_to_h2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
    asm("{\n .reg .b16 a, b;\n mov.b32 {a, b}, %2;\n"
        " cvt.rn.f16x2.e4m3x2 %0, a;\n cvt.rn.f16x2.e4m3x2 %1, b;\n}\n"
        : "=r"(lo), "=r"(hi)
        : "r"(w));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    return __byte_perm(a, b, sel);
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    return h2_as_u32(__floats2half2_rn(lo, hi));
}

// nibble pairs (x bits 0-3 and 16-19) -> f16x2 codes 0..15, exact:
// 0x6400 | c is the half 1024 + c; subtracting 1024 is exact.
__device__ __forceinline__ uint32_t nib2_to_h2(uint32_t x) {
    const uint32_t magic = (x & 0x000F000Fu) | 0x64006400u;
    return h2_as_u32(__hsub2(u32_as_h2(magic), u32_as_h2(0x64006400u)));
}

// high nibbles (x bits 4-7 and 20-23) -> f16x2 codes, exact and shift-free:
// 0x5400 is 64 with a mantissa step of 1/16, so 0x5400 | (c << 4) is 64 + c.
__device__ __forceinline__ uint32_t nib2hi_to_h2(uint32_t x) {
    const uint32_t magic = (x & 0x00F000F0u) | 0x54005400u;
    return h2_as_u32(__hsub2(u32_as_h2(magic), u32_as_h2(0x54005400u)));
}

// dequant v = code * scale + zero in fp16 arithmetic (two roundings, as the
// reference's _dequant_int4_per_token does in fp16)
__device__ __forceinline__ uint32_t dq_h2(uint32_t codes, uint32_t s2, uint32_t z2) {
    return h2_as_u32(__hadd2(__hmul2(u32_as_h2(codes), u32_as_h2(s2)), u32_as_h2(z2)));
}

__device__ __forceinline__ float quad_max(float v) {
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
__device__ __forceinline__ float quad_min(float v) {
    v = fminf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    return fminf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
}
// (value, index) max with earliest index on ties; index -1 = none
__device__ __forceinline__ void argmax_merge(float& v, int& i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 >= 0 && (i < 0 || i2 < i))) {
        v = v2;
        i = i2;
    }
}
__device__ __forceinline__ void quad_argmax(float& v, int& i) {
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
        argmax_merge(v, i, v2, i2);
    }
}

// Per-warp online-softmax state for q head r (quad-shared max) plus the O^T
// accumulators of heads 2c, 2c+1 and the spike trackers.
template <int D>
struct WarpState {
    static constexpr int MT = D / 16;   // PV m-tiles
    float o[MT][4];
    float m;        // running max of head r (natural-log units)
    float l;        // partial denominator (this lane's tokens)
    float z;        // partial sum of p * zero (per-token INT4 zero folded out of V)
    float mn;       // min near/decode score, head r
    float mf;       // max far score, head r
    int af;         // argmax far (far-local index), head r

    __device__ __forceinline__ void init() {
#pragma unroll
        for (int i = 0; i < MT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
        m = -INFINITY;
        l = 0.f;
        z = 0.f;
        mn = INFINITY;
        mf = -INFINITY;
        af = -1;
    }

    // online-softmax update with this lane's N scores of head r (masked =
    // -inf); returns the unnormalised probabilities in p[].
    template <int N>
    __device__ __forceinline__ void softmax_step(const float (&s)[N], float (&p)[N], int lane) {
        float lm = s[0];
#pragma unroll
        for (int j = 1; j < N; ++j) lm = fmaxf(lm, s[j]);
        const float tmax = quad_max(lm);
        const bool up = tmax > m;
        if (__any_sync(0xffffffffu, up)) {
            const float mnew = up ? tmax : m;
            const float alpha = (m == -INFINITY) ? 0.f : exp2f((m - mnew) * kLog2e);
            l *= alpha;
            z *= alpha;
            m = mnew;
            const int c = lane & 3;
            const float a0 = __shfl_sync(0xffffffffu, alpha, (2 * c) * 4);
            const float a1 = __shfl_sync(0xffffffffu, alpha, (2 * c + 1) * 4);
#pragma unroll
            for (int i = 0; i < MT; ++i) {
                o[i][0] *= a0;
                o[i][1] *= a1;
                o[i][2] *= a0;
                o[i][3] *= a1;
            }
        }
        const float mb = m * kLog2e;
#pragma unroll
        for (int j = 0; j < N; ++j) {
            p[j] = exp2f(fmaf(s[j], kLog2e, -mb));   // s = -inf -> 0
            l += p[j];
        }
    }
};

}  // namespace fkvdev

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA, non-tensor, no multicast) primitives
// ---------------------------------------------------------------------------
namespace fkvdev {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` with an iteration limit; false = gave up.
constexpr uint32_t kWaitLimit = 1u << 26;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// global -> shared bulk copy completing on `bar` (bytes and both addresses
// multiples of 16)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace fkvdev
