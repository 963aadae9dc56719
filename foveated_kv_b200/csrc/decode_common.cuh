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
    // -inf) whose maximum is lm; returns the unnormalised probabilities in
    // p[].  The running max m is raised (and l, z, o rescaled) only when the
    // tile's max exceeds it by more than kLazyNats: numerator and
    // denominator always share m, so the result is unchanged, and
    // p = exp(s - m) stays below e^kLazyNats (fp16-safe as P and p*scale).
    static constexpr float kLazyNats = 8.f;
    template <int N>
    __device__ __forceinline__ void softmax_step(const float (&s)[N], float (&p)[N], float lm,
                                                 int lane) {
        const float tmax = quad_max(lm);
        const bool up = tmax > m + kLazyNats;
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
    template <int N>
    __device__ __forceinline__ void softmax_step(const float (&s)[N], float (&p)[N], int lane) {
        float lm = s[0];
#pragma unroll
        for (int j = 1; j < N; ++j) lm = fmaxf(lm, s[j]);
        softmax_step(s, p, lm, lane);
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
// kWaitLimit is the default limit of the progress waits (a caller may lower
// it per launch) and the fixed limit of the clean-up waits that let copies
// and tensor-core work in flight finish before a CTA exits.
constexpr uint32_t kWaitLimit = 1u << 26;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint32_t limit = kWaitLimit) {
    for (uint32_t i = 0; i < limit; ++i)
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

// ---------------------------------------------------------------------------
// 5th-generation tensor core (tcgen05) primitives: tensor memory (TMEM)
// allocation, single-thread MMA issue with shared-memory descriptors, commit
// to an mbarrier, TMEM -> register loads; tensor-map TMA loads (no multicast)
// ---------------------------------------------------------------------------
namespace fkvdev {

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// 2-D tiled tensor-map load of box (x, y) into shared memory (x = 0 here, so
// the innermost coordinate is always 16-byte aligned)
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// generic-proxy shared-memory writes -> visible to the async proxy (tensor
// core operand reads, TMA writes)
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

// whole-warp TMEM allocation of `cols` columns (power of two >= 32); the
// TMEM address is written to *dst
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(dst)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(cols)
                 : "memory");
}

// Shared-memory matrix descriptor of a K-major operand stored as rows of 128
// bytes in the 128-byte swizzle (16-byte chunk c of row r at c ^ (r & 7),
// 8-row groups 1024 bytes apart, tile base 1024-byte aligned).  Fields:
// start address >> 4 (bits 0-13), leading offset (16-29, unused for this
// layout), stride offset 1024 >> 4 (32-45), descriptor version 1 (46),
// layout 2 = 128-byte swizzle (61-63).  Advancing K by 32 bytes inside the
// swizzle row adds 2 to the start address field.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f8f6f4, A and B E4M3 (format 0), both
// K-major, f32 accumulator (bits 4-5 = 1), N >> 3 at bits 17-22, M >> 4 at
// bits 24-28.
__host__ __device__ constexpr uint32_t f8_idesc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem desc] . B[smem desc]^T, issued by one thread
__device__ __forceinline__ void umma_f8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// arrive once on `bar` when every tcgen05 operation this thread issued so far
// has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
            smem_u32(bar))
        : "memory");
}

// warp loads of TMEM lanes 32*(warp%4) + lane, N consecutive 32-bit columns
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
          "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
          "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

}  // namespace fkvdev

// ---------------------------------------------------------------------------
// Thread-block cluster primitives: cluster barrier (all threads of every CTA
// of the cluster, whole warps), distributed shared memory addressing and
// loads / atomics into a peer CTA's shared memory.
// ---------------------------------------------------------------------------
namespace fkvdev {

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t peer_smem(const void* local, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(out) : "r"(smem_u32(local)), "r"(rank));
    return out;
}
__device__ __forceinline__ float ld_peer_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ int ld_peer_s32(uint32_t addr) {
    int v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];\n" : "=r"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t atom_add_peer(uint32_t addr, uint32_t v) {
    uint32_t old;
    asm volatile("atom.shared::cluster.add.u32 %0, [%1], %2;\n" : "=r"(old) : "r"(addr), "r"(v) : "memory");
    return old;
}

}  // namespace fkvdev
