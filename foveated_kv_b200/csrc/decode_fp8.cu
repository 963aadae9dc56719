// Fused two-tier decode attention (fp8 E4M3 K / INT4 V far tier) with spike
// emission, split-K over the concatenated [near | far | decode] sequence and
// the split combine done by the last CTA of each (b, kv-head, head-group).
//
// Semantics follow kernel foveated_2tier (csrc/kernels/foveated_attn.metal:181-432
// of the reference): q pre-scaled by 1/sqrt(D) in fp32, near rows bounded by
// near_valid[b,h] read once per launch, spike flag = max_far > min_near + margin
// with the earliest far index on ties, decode-buffer scores feeding min_near.
// Unlike the Metal kernel every (b, kv head) is read once for all its q heads
// (GQA group on the tensor-core M dimension) and no score-gated V skip is
// applied (the output matches dequantise-then-attend without the exp(-16) cut).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "decode_common.cuh"
#include "fkv_common.h"

using namespace fkvdev;

namespace {

constexpr int kThreads = 5 * 32;   // 4 consumer warps + 1 producer warp
constexpr int kTile = 16;

struct DecodeParams {
    const uint16_t* near_k;
    const uint16_t* near_v;
    const int32_t* near_valid;
    const uint8_t* far_k;
    const uint8_t* far_v;
    const uint16_t* v_scale;
    const uint16_t* v_zero;
    const uint16_t* q;
    const uint16_t* dec_k;
    const uint16_t* dec_v;
    uint16_t* out;
    int32_t* flags;
    int32_t* tokens;
    float* part;          // sequence-split records (nullptr = final output)
    int32_t* part_arg;
    int32_t far_offset;
    float* ws;            // split records
    int32_t* tickets;     // one counter per (stream, head group)
    int32_t* status;      // sticky kernel status word (0 = ok)
    uint32_t wait_limit;  // iteration limit of the progress waits
    int test_stall;       // 1: consumers first wait on a barrier nothing completes
    // TurboQuant far tier (far_k = 2-bit key codes, far_v = 2-bit value codes,
    // v_scale = per-32-dim value scales)
    const uint8_t* k_signs;
    const uint16_t* k_norm;
    const uint16_t* k_gamma;
    const float* centroids;
    const float* qproj;   // (B*Hq, 2D) f32: q Pi^T | q S^T, written by turbo_qproj_kernel
    const float* turbo_pi;
    const float* turbo_s;
    float qjl_coef;
    int B, Hq, Hk, G, HG, Np, F, n_dec, dec_stride, splits;
    int csize, groups;    // cluster mode: CTAs per cluster, clusters per (stream, head group)
    int near_w, far_w;    // cost units of an fp16 near / decode token and of a far token
    float margin, qscale;
};

constexpr int kTurbo = -1;   // VG value selecting the TurboQuant far tier

// Tensor maps of the tier tensors read with tiled TMA copies in the 128-byte
// swizzle: far K codes as (B*Hk*F, D) bytes in 128-row boxes (tensor-core
// path only), near tier and decode buffer as (rows, D) fp16 in boxes of 64
// rows x 64 halves (one box per 128-byte half row).
struct TMaps {
    CUtensorMap far_k;
    CUtensorMap near_k, near_v;
    CUtensorMap dec_k, dec_v;
};
constexpr int kHalfBox = 64 * 128;   // bytes of one 64-row x 128-byte fp16 box

// record = merged state of up to 8 q heads over a token range
template <int D>
struct RecLayout {
    static constexpr int M = 0, L = 8, MN = 16, MF = 24, AF = 32, O = 40;
    static constexpr int SIZE = 40 + 8 * D;   // floats
};

// q pieces of the tensor-core far path, built by one of two warps (half of
// the NH heads each; lane l covers dims [4l, 4l + 4)).  With e = 2^E chosen
// so that max|q| e over the CTA's heads lies in [128, 256) (both warps compute
// the same maximum), piece 0 = e4m3(q e) and piece j+1 = e4m3(16 (r_j -
// piece_j)) of the residual r_j; then q = sum_j piece_j 16^-j / e up to 2^-16
// relative per element, and a score is (acc_0 + acc_1/16 + acc_2/256 +
// acc_3/4096) / e.  Piece j of head hh is row j*NH + hh of the B operand
// (K-major rows of D bytes in the 128-byte swizzle); *escale = 1/e.
constexpr int kQPieces = 4;

template <int D, int NH>
__device__ __forceinline__ void build_q_pieces(const DecodeParams& p, int s, int hg, int half,
                                               int lane, uint8_t* __restrict__ qb, float* escale) {
    static_assert(D == 128, "tensor-core far path assumes 128-byte K rows");
    const int b = s / p.Hk, h = s % p.Hk;
    const int d0 = 4 * lane;
    float q4[NH][4];
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
        const int g = hg * kHeadsPerTile + hh;
        q4[hh][0] = q4[hh][1] = q4[hh][2] = q4[hh][3] = 0.f;
        if (g < p.G) {
            const uint2 w = __ldg(reinterpret_cast<const uint2*>(
                p.q + ((int64_t)b * p.Hq + (int64_t)h * p.G + g) * D + d0));
            const float2 f01 = __half22float2(u32_as_h2(w.x)), f23 = __half22float2(u32_as_h2(w.y));
            q4[hh][0] = f01.x * p.qscale; q4[hh][1] = f01.y * p.qscale;
            q4[hh][2] = f23.x * p.qscale; q4[hh][3] = f23.y * p.qscale;
        }
    }
    float mx = 0.f;
#pragma unroll
    for (int hh = 0; hh < NH; ++hh)
#pragma unroll
        for (int e = 0; e < 4; ++e) mx = fmaxf(mx, fabsf(q4[hh][e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int ex = 0;
    frexpf(mx, &ex);                                      // mx < 2^ex
    const float sc = mx > 0.f ? ldexpf(1.f, 8 - ex) : 1.f;
    if (half == 0 && lane == 0) *escale = 1.f / sc;       // exact: a power of two
#pragma unroll
    for (int j2 = 0; j2 < NH / 2; ++j2) {
        const int hh = half * (NH / 2) + j2;
        float rv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) rv[e] = (half ? q4[NH / 2 + j2][e] : q4[j2][e]) * sc;
#pragma unroll
        for (int j = 0; j < kQPieces; ++j) {
            // hardware conversions: f32 pairs -> E4M3x2 (round to nearest
            // even, saturating) and back E4M3x2 -> f16x2 (exact)
            uint16_t p01, p23;
            asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;\n" : "=h"(p01) : "f"(rv[0]), "f"(rv[1]));
            asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;\n" : "=h"(p23) : "f"(rv[2]), "f"(rv[3]));
            const float2 b01 = __half22float2(u32_as_h2(e4m3x2_to_h2(p01)));
            const float2 b23 = __half22float2(u32_as_h2(e4m3x2_to_h2(p23)));
            rv[0] = (rv[0] - b01.x) * 16.f;               // exact residuals, scaled up
            rv[1] = (rv[1] - b01.y) * 16.f;
            rv[2] = (rv[2] - b23.x) * 16.f;
            rv[3] = (rv[3] - b23.y) * 16.f;
            const int n = j * NH + hh;                    // B row
            *reinterpret_cast<uint32_t*>(qb + n * 128 + ((((d0 >> 4) ^ (n & 7)) << 4) | (d0 & 15))) =
                (uint32_t)p01 | ((uint32_t)p23 << 16);
        }
    }
}

// q A-fragments of the CTA's head group, one uint4 per (k-step, lane), built
// once by consumer warp 0 into shared memory and read by every consumer warp
template <int D>
__device__ __forceinline__ void build_q_frags(const DecodeParams& p, int s, int hg, int lane,
                                              uint4* __restrict__ qs) {
    const int r = lane >> 2, c = lane & 3;
    const int b = s / p.Hk, h = s % p.Hk;
    const int g = hg * kHeadsPerTile + r;
    constexpr int KC = D / 4;   // dims per lane chunk
    float qv[KC];
    if (g < p.G) {
        const uint16_t* qrow = p.q + ((int64_t)b * p.Hq + (int64_t)h * p.G + g) * D + c * KC;
#pragma unroll
        for (int u = 0; u < KC / 8; ++u) {
            const uint4 w = __ldg(reinterpret_cast<const uint4*>(qrow) + u);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                qv[u * 8 + 2 * e] = __half2float(__ushort_as_half(ws[e] & 0xFFFF)) * p.qscale;
                qv[u * 8 + 2 * e + 1] = __half2float(__ushort_as_half(ws[e] >> 16)) * p.qscale;
            }
        }
    } else {
#pragma unroll
        for (int u = 0; u < KC; ++u) qv[u] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < D / 16; ++j) {
        __half hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            hi[e] = __float2half_rn(qv[4 * j + e]);
            lo[e] = __float2half_rn(qv[4 * j + e] - __half2float(hi[e]));
        }
        qs[j * 32 + lane] = make_uint4(h2_as_u32(__halves2half2(hi[0], hi[1])),
                                       h2_as_u32(__halves2half2(lo[0], lo[1])),
                                       h2_as_u32(__halves2half2(hi[2], hi[3])),
                                       h2_as_u32(__halves2half2(lo[2], lo[3])));
    }
}

// Shared-memory ring: a producer warp streams contiguous token chunks of the
// (b, kv head) stream with bulk copies (TMA, cp.async.bulk) into kStages
// slots; 4 consumer warps take 16-token tiles of each slot.  Slot layout:
// [K rows | V rows]; far stages carry 128 tokens, near / decode stages 64.
constexpr int kConsumerWarps = 4;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kStages = 2;

template <int D, int VG = 0>
struct Ring {
    static constexpr int FAR_TOK = 128;
    static constexpr int NEAR_TOK = 64;
    static constexpr int VOFF = NEAR_TOK * D * 2;        // K region (max of near / far)
    static constexpr int SLOT = VOFF + NEAR_TOK * D * 2;  // + V region
    // per-token scalars of a far stage (INT4 scale / zero, or turbo norm /
    // gamma / value scales / QJL signs), each a 16-byte-aligned covering copy
    static constexpr int SEL = (VG == 0) ? 1 : D / 32;           // halves per token in r0/r1
    static constexpr int SZOFF = VOFF + FAR_TOK * (VG == kTurbo ? D / 4 : D / 2);
    static constexpr int RB0 = FAR_TOK * SEL * 2 + 32;           // region bytes (r0, r1)
    static constexpr int RB2 = FAR_TOK * (D / 32) * 2 + 32;      // turbo value scales
    static constexpr int RB3 = FAR_TOK * (D / 8) + 32;           // turbo signs
    static_assert(SZOFF + 2 * RB0 + (VG == kTurbo ? RB2 + RB3 : 0) <= SLOT, "slot overflow");
    static constexpr int QFRAG = (D / 16) * 32 * 16;            // one set of q fragments
    static constexpr int QOFF = kStages * SLOT;                 // q (+ turbo q Pi^T, q S^T)
    static constexpr int TSUM = QOFF + (VG == kTurbo ? 3 : 1) * QFRAG;   // turbo row sums
    static constexpr int BAROFF = TSUM + (VG == kTurbo ? 64 : 0);        // mbarriers
    static constexpr int MERGEBAR = BAROFF + 2 * kStages * 8;          // 2 split-merge barriers
    static constexpr int STALLBAR = MERGEBAR + 2 * 8;                  // never completed (test hook)
    // cluster mode: per-slot stage headers, the cluster's stage counter (used
    // in rank 0), stages issued, producer done
    static constexpr int CTRL = STALLBAR + 8;
    static constexpr int HDR = CTRL, COUNTER = CTRL + 4 * kStages, ISSUED = COUNTER + 4,
                         PDONE = ISSUED + 4;
    // turbo in cluster mode: q Pi^T | q S^T of the CTA's 8 q heads (f32)
    static constexpr int QPJ = (PDONE + 4 + 15) & ~15;
    static constexpr int BYTES = QPJ + (VG == kTurbo ? kHeadsPerTile * 2 * D * 4 : 0);
    // (+1024 at launch: base alignment slack)
};

// Extra shared memory of the tensor-core far path (placed after the ring's
// layout): the q-piece B operand (1024-byte aligned for the 128-byte
// swizzle), the MMA-done / q-ready / drain mbarriers, the TMEM base address and
// the piece scale.  The dynamic shared memory base is rounded up to 1024 bytes
// in the kernel, hence the slack.
template <int D, int VG>
struct UmLayout {
    using RG = Ring<D, VG>;
    static constexpr int QB = (RG::BYTES + 1023) & ~1023;
    static constexpr int MMAB = QB + 4 * kHeadsPerTile * 128;   // kStages MMA-done barriers
    static constexpr int QREADY = MMAB + kStages * 8;
    static constexpr int DRAIN = QREADY + 8;
    static constexpr int TADDR = DRAIN + 8;
    static constexpr int ESC = TADDR + 4;                        // piece scale
    static constexpr int BYTES = ESC + 4 + 1024;
    static constexpr uint32_t TMEM_COLS = 64;   // kStages x 32 score columns
    static_assert(RG::SLOT % 1024 == 0, "ring slots must keep 1024-byte alignment");
    static_assert(MMAB < QREADY && QREADY < DRAIN && DRAIN < TADDR && TADDR < ESC && ESC < BYTES &&
                      TMEM_COLS == kStages * 32,
                  "layout order");
};

// Bytes [b0, b1) of `base` (an array of `total` bytes) into shared `dst`,
// which receives the 16-byte-aligned covering range starting at b0 & ~15: a
// bulk copy for the part inside the array's last full 16 bytes, plain loads
// for a ragged end of the array.  Returns the bulk bytes (for expect_tx).
__device__ __forceinline__ uint32_t copy_covering(uint8_t* dst, const uint8_t* base, int64_t total,
                                                  int64_t b0, int64_t b1, uint64_t* bar) {
    const int64_t a0 = b0 & ~(int64_t)15;
    const int64_t a1 = (b1 + 15) & ~(int64_t)15;
    const int64_t bulk_end = min(a1, total & ~(int64_t)15);
    uint32_t tx = 0;
    if (bulk_end > a0) {
        bulk_g2s(dst, base + a0, (uint32_t)(bulk_end - a0), bar);
        tx = (uint32_t)(bulk_end - a0);
    }
    for (int64_t x = max(a0, bulk_end); x < b1; ++x) dst[x - a0] = base[x];
    return tx;
}

struct Segs {
    int a[3], e[3], n[3];   // tier-local [a, e) and stage counts: near, far, decode
};

template <int D>
__device__ __forceinline__ void stage_at(const Segs& sg, int k, int& seg, int& start, int& cnt) {
    constexpr int NT = Ring<D>::NEAR_TOK, FT = Ring<D>::FAR_TOK;
    if (k < sg.n[0]) {
        seg = 0;
        start = sg.a[0] + k * NT;
        cnt = min(NT, sg.e[0] - start);
    } else if (k < sg.n[0] + sg.n[1]) {
        seg = 1;
        start = sg.a[1] + (k - sg.n[0]) * FT;
        cnt = min(FT, sg.e[1] - start);
    } else {
        seg = 2;
        start = sg.a[2] + (k - sg.n[0] - sg.n[1]) * NT;
        cnt = min(NT, sg.e[2] - start);
    }
}

// ---- one 16-token tile of an fp16 stage (near tier or decode buffer) ----
// The stage holds each of K and V as 128-byte half rows of 64 tokens in the
// 128-byte swizzle: 16-byte chunk j of token u's 2D-byte row sits at half
// j / 8, chunk (j % 8) ^ (u % 8).  The B-fragment reads of K (lane (r, c):
// token r, bytes [c*D/2, (c+1)*D/2)) are then spread over all banks.
__device__ __forceinline__ int sw128_off(int u, int j) {
    return (j >> 3) * kHalfBox + u * 128 + (((j & 7) ^ (u & 7)) << 4);
}

template <int D>
__device__ __forceinline__ void fp16_tile(const uint8_t* __restrict__ kbuf,
                                          const uint8_t* __restrict__ vbuf, int u0, int cnt,
                                          int lane, const uint4* __restrict__ qs,
                                          WarpState<D>& st) {
    constexpr int KW = D / 8;      // u32 words per lane K chunk (D/4 halves)
    constexpr int VW = D / 16;     // u32 words per lane V chunk (D/8 halves)
    const int r = lane >> 2, c = lane & 3;
    uint32_t kr[2][KW];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
        const int u = u0 + 8 * n + r;
#pragma unroll
        for (int x = 0; x < KW / 4; ++x) {
            const uint4 w = *reinterpret_cast<const uint4*>(kbuf + sw128_off(u, c * (KW / 4) + x));
            kr[n][4 * x] = w.x; kr[n][4 * x + 1] = w.y; kr[n][4 * x + 2] = w.z; kr[n][4 * x + 3] = w.w;
        }
    }
    uint32_t vr[4][VW];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int u = u0 + (e >> 1) * 8 + 2 * c + (e & 1);
        const bool ok = u < cnt;
#pragma unroll
        for (int x = 0; x < VW / 4; ++x) {
            const uint4 w = ok ? *reinterpret_cast<const uint4*>(vbuf + sw128_off(u, r * (VW / 4) + x))
                               : make_uint4(0, 0, 0, 0);
            vr[e][4 * x] = w.x; vr[e][4 * x + 1] = w.y; vr[e][4 * x + 2] = w.z; vr[e][4 * x + 3] = w.w;
        }
    }
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int j = 0; j < D / 16; ++j) {
        const uint4 qv = qs[j * 32 + lane];
        const uint32_t qa[4] = {qv.x, qv.y, qv.z, qv.w};
        mma16816(sc[0], qa, kr[0][2 * j], kr[0][2 * j + 1]);
        mma16816(sc[1], qa, kr[1][2 * j], kr[1][2 * j + 1]);
    }
    float s[4], pr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int u = u0 + (j >> 1) * 8 + 2 * c + (j & 1);
        const float v = sc[j >> 1][j & 1] + sc[j >> 1][2 + (j & 1)];
        s[j] = u < cnt ? v : -INFINITY;
        if (u < cnt) st.mn = fminf(st.mn, v);
    }
    st.softmax_step(s, pr, lane);
    const uint32_t pb0 = pack_h2(pr[0], pr[1]);
    const uint32_t pb1 = pack_h2(pr[2], pr[3]);
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
        uint32_t a[4];
        a[0] = prmt(vr[0][i], vr[1][i], 0x5410);
        a[1] = prmt(vr[0][i], vr[1][i], 0x7632);
        a[2] = prmt(vr[2][i], vr[3][i], 0x5410);
        a[3] = prmt(vr[2][i], vr[3][i], 0x7632);
        mma16816(st.o[i], a, pb0, pb1);
    }
}

// scale/zero of the 4 V tokens a lane feeds into the PV product, packed
// (scale | zero << 16); loaded one stage ahead from global memory
template <int D, int VG>
__device__ __forceinline__ void load_sz(const uint16_t* __restrict__ sc,
                                        const uint16_t* __restrict__ ze, int u0, int cnt,
                                        int lane, uint32_t (&sz)[4]) {
    const int r = lane >> 2, c = lane & 3;
    constexpr int EL = (VG == 0) ? 1 : D / VG;   // values per token
    const int grp = (VG == 0) ? 0 : (r * (D / 8)) / (VG == 0 ? 1 : VG);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int u = u0 + (e >> 1) * 8 + 2 * c + (e & 1);
        sz[e] = u < cnt ? ((uint32_t)sc[u * EL + grp] | ((uint32_t)ze[u * EL + grp] << 16)) : 0u;
    }
}

// INT4 V words of NT far tiles in the V^T A-fragment order (lane r: dims
// [r*D/8, (r+1)*D/8) of tokens u0[t] + {2c, 2c+1, 8+2c, 9+2c})
template <int D, int NT>
__device__ __forceinline__ void load_far_v(const uint8_t* __restrict__ vbuf, const int (&u0)[NT],
                                           int cnt, int lane,
                                           uint32_t (&vr)[NT][4][(D / 16 + 3) / 4]) {
    constexpr int VB = D / 16;    // bytes of INT4 V per lane per token (D/8 dims)
    const int r = lane >> 2, c = lane & 3;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int u = u0[t] + (e >> 1) * 8 + 2 * c + (e & 1);
            const bool ok = u < cnt;
            const uint8_t* src = vbuf + u * (D / 2) + r * VB;
            if constexpr (VB == 8) {
                const uint2 w = ok ? *reinterpret_cast<const uint2*>(src) : make_uint2(0, 0);
                vr[t][e][0] = w.x;
                vr[t][e][1] = w.y;
            } else {
                vr[t][e][0] = ok ? *reinterpret_cast<const uint32_t*>(src) : 0u;
            }
        }
    }
}

// Masking, spike tracking, online softmax and the P.V product of NT far
// tiles whose raw scores `sv` are in the S C-fragment layout (lane (r, c):
// head r, tokens u0[t] + {2c, 2c+1, 8+2c, 9+2c}) and whose V words are in vr.
template <int D, int VG, int NT, bool CL = false>
__device__ __forceinline__ void far_tail(const float (&sv)[4 * NT],
                                         const uint32_t (&vr)[NT][4][(D / 16 + 3) / 4],
                                         const int (&u0)[NT], int cnt, int gbase, int lane,
                                         const uint32_t (&sz)[NT][4], WarpState<D>& st) {
    const int c = lane & 3;
    float s[4 * NT], pr[4 * NT];
    float lm = -INFINITY;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int u = u0[t] + (j >> 1) * 8 + 2 * c + (j & 1);
            s[4 * t + j] = u < cnt ? sv[4 * t + j] : -INFINITY;
            lm = fmaxf(lm, s[4 * t + j]);
        }
    }
    // spike tracker: the lane's values are in token order, so the earliest
    // index of a new strict maximum is the first j holding it (rare branch)
    // (stages may arrive out of token order in cluster mode: there an equal
    // maximum replaces the tracked one when its index is lower)
    if (CL ? (lm >= st.mf && lm != -INFINITY) : lm > st.mf) {
        int jj = 0;
#pragma unroll
        for (int j = 4 * NT - 1; j >= 0; --j)
            if (s[j] == lm) jj = j;
        const int ut = (NT > 1 && jj >= 4) ? u0[NT - 1] : u0[0];
        const int idx = gbase + ut + ((jj & 3) >> 1) * 8 + 2 * c + (jj & 1);
        if (!CL || lm > st.mf || idx < st.af) {
            st.mf = lm;
            st.af = idx;
        }
    }
    st.softmax_step(s, pr, lm, lane);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        uint32_t pb0, pb1;
        if constexpr (VG == 0) {
            // per-token scale folded into P, zero into a running sum p * z:
            // sum_t p_t (c_t s_t + z_t) = sum_t (p_t s_t) c_t + sum_t p_t z_t
            float ps[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(u32_as_h2(sz[t][e]));   // (scale, zero)
                ps[e] = pr[4 * t + e] * f.x;
                st.z = fmaf(pr[4 * t + e], f.y, st.z);
            }
            pb0 = pack_h2(ps[0], ps[1]);
            pb1 = pack_h2(ps[2], ps[3]);
#pragma unroll
            for (int i = 0; i < D / 16; ++i) {
                const int wi = i >> 2, bi = i & 3;
                const uint32_t sel = (uint32_t)bi | ((uint32_t)(4 + bi) << 8);
                const uint32_t xab = prmt(vr[t][0][wi], vr[t][1][wi], sel);
                const uint32_t xcd = prmt(vr[t][2][wi], vr[t][3][wi], sel);
                uint32_t a[4];
                a[0] = nib2_to_h2(xab);
                a[1] = nib2hi_to_h2(xab);
                a[2] = nib2_to_h2(xcd);
                a[3] = nib2hi_to_h2(xcd);
                mma16816(st.o[i], a, pb0, pb1);
            }
        } else {
            pb0 = pack_h2(pr[4 * t + 0], pr[4 * t + 1]);
            pb1 = pack_h2(pr[4 * t + 2], pr[4 * t + 3]);
            const uint32_t sAB = (sz[t][0] & 0xFFFFu) | (sz[t][1] << 16);
            const uint32_t zAB = (sz[t][0] >> 16) | (sz[t][1] & 0xFFFF0000u);
            const uint32_t sCD = (sz[t][2] & 0xFFFFu) | (sz[t][3] << 16);
            const uint32_t zCD = (sz[t][2] >> 16) | (sz[t][3] & 0xFFFF0000u);
#pragma unroll
            for (int i = 0; i < D / 16; ++i) {
                const int wi = i >> 2, bi = i & 3;
                const uint32_t sel = (uint32_t)bi | ((uint32_t)(4 + bi) << 8);
                const uint32_t xab = prmt(vr[t][0][wi], vr[t][1][wi], sel);
                const uint32_t xcd = prmt(vr[t][2][wi], vr[t][3][wi], sel);
                uint32_t a[4];
                a[0] = dq_h2(nib2_to_h2(xab), sAB, zAB);
                a[1] = dq_h2(nib2hi_to_h2(xab), sAB, zAB);
                a[2] = dq_h2(nib2_to_h2(xcd), sCD, zCD);
                a[3] = dq_h2(nib2hi_to_h2(xcd), sCD, zCD);
                mma16816(st.o[i], a, pb0, pb1);
            }
        }
    }
}

// ---- NT 16-token tiles of an fp8 / INT4 far stage, processed jointly ----
// (the tiles' loads, conversions and tensor-core products are interleaved and
// share one online-softmax step, which gives each warp instruction-level
// parallelism at the occupancy the register budget allows)
template <int D, int VG, int NT, bool CL = false>
__device__ __forceinline__ void far_tiles(const uint8_t* __restrict__ kbuf,
                                          const uint8_t* __restrict__ vbuf, const int (&u0)[NT],
                                          int cnt, int gbase, int lane,
                                          const uint4* __restrict__ qs,
                                          const uint32_t (&sz)[NT][4], WarpState<D>& st) {
    constexpr int KW = D / 16;    // u32 words of fp8 K per lane per token (D/4 bytes)
    constexpr int VWN = (D / 16 + 3) / 4;
    const int r = lane >> 2, c = lane & 3;
    uint32_t kr[NT][2][KW];
    uint32_t vr[NT][4][VWN];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int n = 0; n < 2; ++n) {
            const int u = u0[t] + 8 * n + r;
            const uint4* src = reinterpret_cast<const uint4*>(kbuf + u * D + c * (D / 4));
            if constexpr (KW == 8) {
                // odd rows read their second 16 bytes first: conflict-free phases
                const int f = r & 1;
                const uint4 w0 = src[f], w1 = src[f ^ 1];
                const uint4 lo = f ? w1 : w0, hi = f ? w0 : w1;
                kr[t][n][0] = lo.x; kr[t][n][1] = lo.y; kr[t][n][2] = lo.z; kr[t][n][3] = lo.w;
                kr[t][n][4] = hi.x; kr[t][n][5] = hi.y; kr[t][n][6] = hi.z; kr[t][n][7] = hi.w;
            } else {
                const uint4 w = src[0];
                kr[t][n][0] = w.x; kr[t][n][1] = w.y; kr[t][n][2] = w.z; kr[t][n][3] = w.w;
            }
        }
    }
    load_far_v<D, NT>(vbuf, u0, cnt, lane, vr);
    float sc[NT][2][4];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int n = 0; n < 2; ++n) sc[t][n][0] = sc[t][n][1] = sc[t][n][2] = sc[t][n][3] = 0.f;
#pragma unroll
    for (int j = 0; j < D / 16; ++j) {
        const uint4 qv = qs[j * 32 + lane];
        const uint32_t qa[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int n = 0; n < 2; ++n) {
                uint32_t b0, b1;
                e4m3x4_to_h2x2(kr[t][n][j], b0, b1);
                mma16816(sc[t][n], qa, b0, b1);
            }
        }
    }
    float sv[4 * NT];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int j = 0; j < 4; ++j) sv[4 * t + j] = sc[t][j >> 1][j & 1] + sc[t][j >> 1][2 + (j & 1)];
    far_tail<D, VG, NT, CL>(sv, vr, u0, cnt, gbase, lane, sz, st);
}

// ---- far tiles scored on the 5th-generation tensor cores (tcgen05) ----
// The producer lane issues, per 128-token far stage, S^T = K . Qp^T with
// tcgen05.mma kind::f8f6f4: A = the stage's E4M3 K codes exactly as stored
// (128 tokens x D bytes, loaded by a tensor-map TMA copy in the 128-byte
// swizzle), B = Qp, the CTA's q heads split into four E4M3 pieces, f32
// accumulators in tensor memory (TMEM lane = token, column = piece * NH +
// head).  No K conversion runs on the SM cores.  Consumer warp w owns TMEM
// lanes / tokens [32w, 32w + 32): it loads its rows, folds the pieces,
// transposes the scores through shared memory into the S C-fragment layout
// and continues with far_tail (softmax, INT4 V on mma.sync).

// floats per head row of the score transpose buffer (row r at bank offset 8r:
// conflict-free float2 reads)
constexpr int kTsStride = 40;

// Returns false when the MMA-done barrier `mmab` (phase `parity`) timed out.
template <int D, int VG, int NT, int NH>
__device__ __forceinline__ bool far_tiles_um(uint8_t* __restrict__ kbuf,
                                             const uint8_t* __restrict__ vbuf, const int (&u0)[NT],
                                             int cnt, int gbase, int lane, int w, uint32_t taddr,
                                             float escale, uint64_t* mmab, uint32_t parity,
                                             uint32_t limit, const uint32_t (&sz)[NT][4],
                                             WarpState<D>& st) {
    constexpr int VWN = (D / 16 + 3) / 4;
    const int r = lane >> 2, c = lane & 3;
    uint32_t vr[NT][4][VWN];
    load_far_v<D, NT>(vbuf, u0, cnt, lane, vr);   // V loads overlap the MMA wait
    if (!mbar_wait(mmab, parity, limit)) return false;
    tc_fence_after();
    uint32_t acc[kQPieces * NH];
    if constexpr (NH == 4) tmem_ld16(taddr, acc);
    else tmem_ld32(taddr, acc);
    tmem_wait_ld();
    // the stage's K codes were consumed by the MMA: its K region is free for
    // the per-warp transpose [head][token]
    float* tb = reinterpret_cast<float*>(kbuf) + w * (NH * kTsStride);
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
        float v = __uint_as_float(acc[hh]);
        v = fmaf(__uint_as_float(acc[NH + hh]), 0.0625f, v);
        v = fmaf(__uint_as_float(acc[2 * NH + hh]), 0.00390625f, v);
        v = fmaf(__uint_as_float(acc[3 * NH + hh]), 0.000244140625f, v);
        tb[hh * kTsStride + lane] = v * escale;
    }
    __syncwarp();
    float sv[4 * NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int x = 0; x < 2; ++x) {
            float2 v2 = make_float2(0.f, 0.f);      // rows r >= NH: no q head (zero q)
            if (r < NH)
                v2 = *reinterpret_cast<const float2*>(tb + r * kTsStride + (u0[t] & 31) + 8 * x + 2 * c);
            sv[4 * t + 2 * x] = v2.x;
            sv[4 * t + 2 * x + 1] = v2.y;
        }
    }
    far_tail<D, VG, NT>(sv, vr, u0, cnt, gbase, lane, sz, st);
    return true;
}

// ---------------------------------------------------------------------------
// TurboQuant far tier: scores directly on codes
// ---------------------------------------------------------------------------
// far score = (|k| * <q Pi^T, c[idx]> + qjl_coef/D * gamma * <q S^T, sign>) / sqrt(D)
// (foveated_attn.metal:486-521,684-688).  c[idx] is written through the
// code's bits b0 (low), b1 as c0 + (c1-c0) b0 + (c2-c0) b1 + ((c3-c2)-(c1-c0))
// b0 b1 (the last term is zero for the symmetric Lloyd-Max centroids and is
// then skipped: two products per 16 dims instead of three) and sign as
// 2[bit] - 1, so the tensor cores only see {0, 1} B fragments (exact in f16)
// against hi/lo-split q Pi^T and q S^T fragments; the centroids and sums are
// applied to the fp32 results.  Turbo K dimension permutation: k-step j, lane
// c covers dims 4(4j+c) .. 4(4j+c)+3 = code byte 4j+c of the token row.

// q Pi^T and q S^T for every (b, q head), f32 (the reference does these two
// products with host matmuls, foveated_attn.cpp:419-421).  A tiny GEMM
// (B*Hq x D) . (D x 2D): each block stages kQpRows rows of [Pi; S] and kQpHeads
// q vectors in shared memory with one round of 16-byte loads, then each
// thread computes one (head, output) dot product.  Grid (2D / kQpRows,
// ceil(B*Hq / kQpHeads)): wide, so the latency is a couple of load rounds.
constexpr int kQpRows = 16, kQpHeads = 8, kQpThreads = kQpRows * kQpHeads;

template <int D>
__global__ void __launch_bounds__(kQpThreads)
    turbo_qproj_kernel(const uint16_t* __restrict__ q, const float* __restrict__ Pi,
                       const float* __restrict__ Sm, float* __restrict__ out, int BH) {
    __shared__ __align__(16) float mrow[kQpRows][D + 4];
    __shared__ __align__(16) float qv[kQpHeads][D + 4];
    const int o0 = blockIdx.x * kQpRows, h0 = blockIdx.y * kQpHeads;
    const int tid = threadIdx.x;
    // Pi and S are constants: staged while the previous kernel of the stream
    // may still run (this grid is launched with programmatic serialization)
    for (int i = tid; i < kQpRows * D / 4; i += kQpThreads) {
        const int r = i / (D / 4), c4 = i % (D / 4), o = o0 + r;
        const float* src = (o < D ? Pi + (int64_t)o * D : Sm + (int64_t)(o - D) * D) + 4 * c4;
        *reinterpret_cast<float4*>(&mrow[r][4 * c4]) = __ldg(reinterpret_cast<const float4*>(src));
    }
    // q may be the previous kernel's output: wait for it to complete; then
    // the decode kernel launched next may start (only its warp that reads
    // these projections waits for this grid; its other reads are ordered
    // after this grid's wait)
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    for (int i = tid; i < kQpHeads * D / 8; i += kQpThreads) {
        const int j = i / (D / 8), c8 = i % (D / 8);
        uint4 w = make_uint4(0, 0, 0, 0);
        if (h0 + j < BH) w = __ldg(reinterpret_cast<const uint4*>(q + (int64_t)(h0 + j) * D) + c8);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(u32_as_h2(ws[e]));
            qv[j][8 * c8 + 2 * e] = f.x;
            qv[j][8 * c8 + 2 * e + 1] = f.y;
        }
    }
    __syncthreads();
    const int j = tid / kQpRows, r = tid % kQpRows;
    float acc = 0.f;
#pragma unroll 16
    for (int i = 0; i < D; ++i) acc = fmaf(qv[j][i], mrow[r][i], acc);
    if (h0 + j < BH) out[(int64_t)(h0 + j) * 2 * D + o0 + r] = acc;
}

// hi/lo fragments of q Pi^T and q S^T in the turbo permutation + per-head sums
// (qsh != nullptr: the projections of the CTA's 8 heads are in shared memory,
// head r at qsh + r * 2D, as the cluster mode computes them)
template <int D>
__device__ __forceinline__ void build_turbo_frags(const DecodeParams& p, int s, int hg, int lane,
                                                  uint4* __restrict__ qr, uint4* __restrict__ qk,
                                                  float* __restrict__ sums,
                                                  const float* qsh = nullptr) {
    const int r = lane >> 2, c = lane & 3;
    const int b = s / p.Hk, h = s % p.Hk;
    const int g = hg * kHeadsPerTile + r;
    const float* src = g >= p.G ? nullptr
                       : qsh != nullptr ? qsh + r * 2 * D
                                        : p.qproj + ((int64_t)b * p.Hq + (int64_t)h * p.G + g) * 2 * D;
    float sr = 0.f, sk = 0.f;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
        uint4* dst = which ? qk : qr;
#pragma unroll
        for (int j = 0; j < D / 16; ++j) {
            __half hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int o = which * D + 4 * (4 * j + c) + e;
                const float v = src == nullptr ? 0.f : qsh != nullptr ? src[o] : __ldg(src + o);
                if (which) sk += v; else sr += v;
                hi[e] = __float2half_rn(v);
                lo[e] = __float2half_rn(v - __half2float(hi[e]));
            }
            dst[j * 32 + lane] = make_uint4(h2_as_u32(__halves2half2(hi[0], hi[1])),
                                            h2_as_u32(__halves2half2(lo[0], lo[1])),
                                            h2_as_u32(__halves2half2(hi[2], hi[3])),
                                            h2_as_u32(__halves2half2(lo[2], lo[3])));
        }
    }
    sr = quad_sum(sr);
    sk = quad_sum(sk);
    if (c == 0) {
        sums[r] = sr;
        sums[8 + r] = sk;
    }
}

// norm | gamma << 16 and the value group scale of the lane's 4 PV tokens
template <int D>
__device__ __forceinline__ void load_turbo_sz(const uint16_t* __restrict__ nm,
                                              const uint16_t* __restrict__ gm,
                                              const uint16_t* __restrict__ vsc, int u0, int cnt,
                                              int lane, uint32_t (&ng)[4], uint32_t (&vs)[2]) {
    const int r = lane >> 2, c = lane & 3;
    const int grp = (r * (D / 8)) / 32;
    uint16_t sv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int u = u0 + (e >> 1) * 8 + 2 * c + (e & 1);
        const bool ok = u < cnt;
        ng[e] = ok ? ((uint32_t)nm[u] | ((uint32_t)gm[u] << 16)) : 0u;
        sv[e] = ok ? vsc[u * (D / 32) + grp] : (uint16_t)0;
    }
    vs[0] = (uint32_t)sv[0] | ((uint32_t)sv[1] << 16);
    vs[1] = (uint32_t)sv[2] | ((uint32_t)sv[3] << 16);
}

// {0,1} f16 pairs: bit 0 and bit 16 of x -> 0x3C00 (1.0) in the matching half
__device__ __forceinline__ uint32_t bits2_to_h2(uint32_t x) { return (x & 0x00010001u) * 0x3C00u; }

template <int D, bool CL = false>
__device__ __forceinline__ void turbo_tile(const uint8_t* __restrict__ sgn,
                                           const uint8_t* __restrict__ kbuf,
                                           const uint8_t* __restrict__ vbuf, int u0, int cnt,
                                           int64_t srow0, int gbase, int lane,
                                           const uint4* __restrict__ qr,
                                           const uint4* __restrict__ qk, const float (&cf)[6],
                                           float sum_r, float sum_k, const uint32_t (&ng)[4],
                                           const uint32_t (&vsc)[2], WarpState<D>& st) {
    constexpr int IW = D / 16;    // u32 words of 2-bit key codes per token (D/4 bytes)
    constexpr int SB = D / 8;     // sign bytes per token
    const int r = lane >> 2, c = lane & 3;
    uint32_t kr[2][IW];
    uint32_t sg[2][SB / 4];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
        const int u = u0 + 8 * n + r;
        const uint4* src = reinterpret_cast<const uint4*>(kbuf + u * (D / 4));
#pragma unroll
        for (int x = 0; x < IW / 4; ++x) {
            const uint4 w4 = src[x];
            kr[n][4 * x] = w4.x; kr[n][4 * x + 1] = w4.y; kr[n][4 * x + 2] = w4.z; kr[n][4 * x + 3] = w4.w;
        }
        const uint8_t* gs = sgn + u * SB;   // may be only 8-byte aligned (D = 64)
#pragma unroll
        for (int x = 0; x < SB / 4; ++x) sg[n][x] = *reinterpret_cast<const uint32_t*>(gs + 4 * x);
    }
    float acc[4][2][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int n = 0; n < 2; ++n) acc[a][n][0] = acc[a][n][1] = acc[a][n][2] = acc[a][n][3] = 0.f;
#pragma unroll
    for (int j = 0; j < D / 16; ++j) {
        const uint4 rv = qr[j * 32 + lane];
        const uint4 kv = qk[j * 32 + lane];
        const uint32_t ar[4] = {rv.x, rv.y, rv.z, rv.w};
        const uint32_t ak[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int n = 0; n < 2; ++n) {
            const uint32_t x = (kr[n][j] >> (8 * c)) & 0xFFu;   // codes of dims 4(4j+c)+0..3
            const uint32_t y01 = x | (x << 14);                 // dim0 -> bits 0-1, dim1 -> 16-17
            const uint32_t y23 = (x >> 4) | (x << 10);          // dim2 -> bits 0-1, dim3 -> 16-17
            mma16816(acc[0][n], ar, bits2_to_h2(y01), bits2_to_h2(y23));             // low bit
            mma16816(acc[1][n], ar, bits2_to_h2(y01 >> 1), bits2_to_h2(y23 >> 1));   // high bit
            if (cf[3] != 0.f)   // both bits (asymmetric centroids only; warp-uniform)
                mma16816(acc[2][n], ar, bits2_to_h2(y01 & (y01 >> 1)), bits2_to_h2(y23 & (y23 >> 1)));
            const int sbyte = 2 * j + (c >> 1);                  // sign byte of these dims
            const uint32_t z = (sg[n][sbyte >> 2] >> (8 * (sbyte & 3) + 4 * (c & 1))) & 0xFu;
            mma16816(acc[3][n], ak, bits2_to_h2(z | (z << 15)), bits2_to_h2((z >> 2) | (z << 13)));
        }
    }
    float s[4], pr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int u = u0 + (j >> 1) * 8 + 2 * c + (j & 1);
        const int n = j >> 1, e = j & 1;
        const float b0 = acc[0][n][e] + acc[0][n][2 + e];
        const float b1 = acc[1][n][e] + acc[1][n][2 + e];
        const float b01 = acc[2][n][e] + acc[2][n][2 + e];
        const float sgn = acc[3][n][e] + acc[3][n][2 + e];
        const float2 f = __half22float2(u32_as_h2(ng[j]));      // (norm, gamma)
        const float mse = fmaf(cf[3], b01, fmaf(cf[2], b1, fmaf(cf[1], b0, cf[0] * sum_r)));
        const float qjl = cf[4] * f.y * fmaf(2.f, sgn, -sum_k);
        const float v = fmaf(f.x, mse, qjl) * cf[5];
        s[j] = u < cnt ? v : -INFINITY;
        if (u < cnt && (v > st.mf || (CL && v == st.mf && gbase + u < st.af))) {
            st.mf = v;
            st.af = gbase + u;
        }
    }
    st.softmax_step(s, pr, lane);
    const uint32_t pb0 = pack_h2(pr[0], pr[1]);
    const uint32_t pb1 = pack_h2(pr[2], pr[3]);
    // value levels {-1, -1/3, 1/3, 1} as f16, selected by prmt
    const uint32_t lut0 = h2_as_u32(__floats2half2_rn(-1.f, -1.f / 3.f));
    const uint32_t lut1 = h2_as_u32(__floats2half2_rn(1.f / 3.f, 1.f));
    uint32_t vw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int u = u0 + (e >> 1) * 8 + 2 * c + (e & 1);
        const uint8_t* src = vbuf + u * (D / 4) + r * (D / 32);
        if constexpr (D == 128) vw[e] = u < cnt ? *reinterpret_cast<const uint32_t*>(src) : 0u;
        else vw[e] = u < cnt ? (uint32_t)*reinterpret_cast<const uint16_t*>(src) : 0u;
    }
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
        const int sh = 8 * (i >> 1) + 4 * (i & 1);
        uint32_t a[4];
#pragma unroll
        for (int half = 0; half < 2; ++half) {        // tokens (A,B) then (C,D)
#pragma unroll
            for (int dd = 0; dd < 2; ++dd) {           // dim d0 then d1
                const uint32_t ca = (vw[2 * half] >> (sh + 2 * dd)) & 3u;
                const uint32_t cb = (vw[2 * half + 1] >> (sh + 2 * dd)) & 3u;
                const uint32_t sel = (ca | (cb << 8)) * 0x22u + 0x1010u;
                const uint32_t lv = prmt(lut0, lut1, sel);
                a[2 * half + dd] = h2_as_u32(__hmul2(u32_as_h2(lv), u32_as_h2(vsc[half])));
            }
        }
        mma16816(st.o[i], a, pb0, pb1);
    }
}

// Cluster mode, TurboQuant: the q Pi^T | q S^T projections of the cluster's
// 8 q heads are computed in slices, rank r taking output columns
// [r * cw, (r + 1) * cw) of the 2D, then gathered from the peers' shared
// memory.  Each output is the same fp32 dot product, in the same order, as
// turbo_qproj_kernel computes.
template <int D>
__device__ __forceinline__ void turbo_qproj_slice(const DecodeParams& p, int s, int hg, int crank,
                                                  float* __restrict__ qpj) {
    const int C = p.csize;
    const int cw = (2 * D + C - 1) / C, c0 = crank * cw;
    const int nc = max(0, min(2 * D, c0 + cw) - c0);
    const int b = s / p.Hk, h = s % p.Hk;
    for (int idx = threadIdx.x; idx < kHeadsPerTile * nc; idx += kConsumerThreads) {
        const int hh = idx / nc, col = c0 + idx % nc;
        const int g = hg * kHeadsPerTile + hh;
        float acc = 0.f;
        if (g < p.G) {
            const uint16_t* qrow = p.q + ((int64_t)b * p.Hq + (int64_t)h * p.G + g) * D;
            const float* mrow = col < D ? p.turbo_pi + (int64_t)col * D : p.turbo_s + (int64_t)(col - D) * D;
#pragma unroll
            for (int i = 0; i < D; i += 8) {
                const uint4 qw = __ldg(reinterpret_cast<const uint4*>(qrow + i));
                const float4 m0 = __ldg(reinterpret_cast<const float4*>(mrow + i));
                const float4 m1 = __ldg(reinterpret_cast<const float4*>(mrow + i + 4));
                const float2 a = __half22float2(u32_as_h2(qw.x)), bq = __half22float2(u32_as_h2(qw.y));
                const float2 cq = __half22float2(u32_as_h2(qw.z)), dq = __half22float2(u32_as_h2(qw.w));
                acc = fmaf(a.x, m0.x, acc); acc = fmaf(a.y, m0.y, acc);
                acc = fmaf(bq.x, m0.z, acc); acc = fmaf(bq.y, m0.w, acc);
                acc = fmaf(cq.x, m1.x, acc); acc = fmaf(cq.y, m1.y, acc);
                acc = fmaf(dq.x, m1.z, acc); acc = fmaf(dq.y, m1.w, acc);
            }
        }
        qpj[hh * 2 * D + col] = acc;
    }
}

template <int D>
__device__ __forceinline__ void turbo_qproj_gather(const DecodeParams& p, int crank,
                                                   float* __restrict__ qpj) {
    const int C = p.csize;
    const int cw = (2 * D + C - 1) / C;
    constexpr int PER = kHeadsPerTile * 2 * D / kConsumerThreads;
    float v[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {   // every load issued before the first store
        const int idx = (int)threadIdx.x + i * kConsumerThreads;
        const int owner = (idx % (2 * D)) / cw;
        v[i] = owner != crank ? ld_peer_f32(peer_smem(qpj + idx, (uint32_t)owner)) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int idx = (int)threadIdx.x + i * kConsumerThreads;
        if ((idx % (2 * D)) / cw != crank) qpj[idx] = v[i];
    }
}

// Merging `n` records of one (stream, head group): per-warp records of one
// CTA (in shared memory) or the split records of all CTAs of the stream (in
// the workspace), then the output or the sequence-split record is emitted.
// merge_heads: the records' scalars are staged in shared memory with one
// round of float4 loads, then 16 threads per head reduce the maxima, the
// weights exp(m_k - M), the denominators and the spike trackers.  The o
// vectors are then accumulated by every thread over its 8 (D = 128) or 4
// (D = 64) contiguous outputs: straight from shared memory for the per-warp
// records, and for the split records with one round of direct loads (few
// records, or few active heads) or through double-buffered bulk copies (TMA)
// of whole records (bandwidth- instead of latency-bound for many splits).
constexpr int kMaxSplits = 64;
constexpr int kDirectMerge = 10;   // split counts merged with direct loads
constexpr int kNarrowLoads = 8;    // records per thread in the few-heads merge
constexpr int kMergeGroup = 8;     // first-level group of the two-level merge
constexpr int kMergeScratch = (kMaxSplits * 40 + kMaxSplits * 8 + 8) * 4;   // bytes

template <bool G>
__device__ __forceinline__ float4 ld4(const float* a) {
    if constexpr (G) return __ldcg(reinterpret_cast<const float4*>(a));
    else return *reinterpret_cast<const float4*>(a);
}

// grec != nullptr: instead of the outputs, the merged record of all 8 heads
// (RecLayout, o unnormalised) is written there -- the first level of a
// two-level merge
template <int D, bool FROM_GLOBAL>
__device__ __forceinline__ void merge_heads(const DecodeParams& p, const float* recs, int n,
                                            int stride, int s, int hg, float* __restrict__ scratch,
                                            float* __restrict__ grec = nullptr) {
    using R = RecLayout<D>;
    static_assert(kConsumerThreads == 128, "merge layout: 16 threads per head");
    const int tid = threadIdx.x;
    const int b = s / p.Hk, h = s % p.Hk;
    float* sc = scratch;                      // [n][40] record scalars
    float* wk = scratch + kMaxSplits * 40;    // [n][8] weights exp(m_k - M)
    float* hl = wk + kMaxSplits * 8;          // [8] L per head
    {
        constexpr int PER = (kMaxSplits * 10 + kConsumerThreads - 1) / kConsumerThreads;
        float4 t[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int i = tid + j * kConsumerThreads;
            if (i < n * 10) t[j] = ld4<FROM_GLOBAL>(recs + (i / 10) * stride + (i % 10) * 4);
        }
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int i = tid + j * kConsumerThreads;
            if (i < n * 10) reinterpret_cast<float4*>(sc)[i] = t[j];
        }
    }
    named_sync(1, kConsumerThreads);
    const int head = tid >> 4, sub = tid & 15;
    float M = -INFINITY;
    for (int k = sub; k < n; k += 16) M = fmaxf(M, sc[k * 40 + R::M + head]);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f, mn = INFINITY, mf = -INFINITY;
    int af = -1;
    for (int k = sub; k < n; k += 16) {
        const float mk = sc[k * 40 + R::M + head];
        const float wgt = (mk == -INFINITY) ? 0.f : exp2f((mk - M) * kLog2e);
        wk[k * 8 + head] = wgt;
        L = fmaf(wgt, sc[k * 40 + R::L + head], L);
        mn = fminf(mn, sc[k * 40 + R::MN + head]);
        argmax_merge(mf, af, sc[k * 40 + R::MF + head], __float_as_int(sc[k * 40 + R::AF + head]));
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
        L += __shfl_xor_sync(0xffffffffu, L, o);
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        const float mf2 = __shfl_xor_sync(0xffffffffu, mf, o);
        const int af2 = __shfl_xor_sync(0xffffffffu, af, o);
        argmax_merge(mf, af, mf2, af2);
    }
    const int g = hg * kHeadsPerTile + head;
    if (sub == 0) {
        hl[head] = L;
        if (grec != nullptr) {
            grec[R::M + head] = M;
            grec[R::L + head] = L;
            grec[R::MN + head] = mn;
            grec[R::MF + head] = mf;
            grec[R::AF + head] = __int_as_float(af);
        } else if (g < p.G) {
            const int64_t bh = (int64_t)b * p.Hq + (int64_t)h * p.G + g;
            if (p.part != nullptr) {
                *reinterpret_cast<float4*>(p.part + bh * (D + 4)) = make_float4(M, L, mn, mf);
                p.part_arg[bh] = af >= 0 ? af + p.far_offset : -1;
            } else {
                p.flags[bh] = (mf > mn + p.margin) ? 1 : 0;
                p.tokens[bh] = af;
            }
        }
    }
    named_sync(1, kConsumerThreads);
}

template <int D>
__device__ __forceinline__ void merge_accumulate(float (&acc)[8 * D / kConsumerThreads],
                                                 const float* rec, float wgt, int e0) {
    using R = RecLayout<D>;
    constexpr int E = 8 * D / kConsumerThreads;
#pragma unroll
    for (int j = 0; j < E / 4; ++j) {
        const float4 v = *reinterpret_cast<const float4*>(rec + R::O + e0 + 4 * j);
        acc[4 * j + 0] = fmaf(wgt, v.x, acc[4 * j + 0]);
        acc[4 * j + 1] = fmaf(wgt, v.y, acc[4 * j + 1]);
        acc[4 * j + 2] = fmaf(wgt, v.z, acc[4 * j + 2]);
        acc[4 * j + 3] = fmaf(wgt, v.w, acc[4 * j + 3]);
    }
}

// thread's E contiguous outputs -> out (fp16, divided by L) or the partial record
template <int D>
__device__ __forceinline__ void merge_emit(const DecodeParams& p, const float (&acc)[8 * D / kConsumerThreads],
                                          int s, int hg, const float* __restrict__ scratch,
                                          float* __restrict__ grec = nullptr) {
    using R = RecLayout<D>;
    constexpr int E = 8 * D / kConsumerThreads;
    const float* hl = scratch + kMaxSplits * 40 + kMaxSplits * 8;
    const int e0 = threadIdx.x * E, head = e0 / D, d0 = e0 % D;
    if (grec != nullptr) {
#pragma unroll
        for (int j = 0; j < E / 4; ++j)
            *reinterpret_cast<float4*>(grec + R::O + e0 + 4 * j) =
                make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
        return;
    }
    const int g = hg * kHeadsPerTile + head;
    if (g >= p.G) return;
    const int b = s / p.Hk, h = s % p.Hk;
    const int64_t bh = (int64_t)b * p.Hq + (int64_t)h * p.G + g;
    if (p.part != nullptr) {
        float* dst = p.part + bh * (D + 4) + 4 + d0;
#pragma unroll
        for (int j = 0; j < E / 4; ++j)
            *reinterpret_cast<float4*>(dst + 4 * j) =
                make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
    } else {
        const float L = hl[head];
        uint32_t hw[E / 2];
#pragma unroll
        for (int x = 0; x < E / 2; ++x)
            hw[x] = pack_h2(L > 0.f ? acc[2 * x] / L : 0.f, L > 0.f ? acc[2 * x + 1] / L : 0.f);
        uint16_t* dst = p.out + bh * D + d0;
        if constexpr (E == 8) *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        else *reinterpret_cast<uint2*>(dst) = make_uint2(hw[0], hw[1]);
    }
}

// the per-warp records of a single-split stream, in shared memory
template <int D>
__device__ __forceinline__ void merge_warps(const DecodeParams& p, const float* recs, int s, int hg,
                                           float* __restrict__ scratch) {
    using R = RecLayout<D>;
    constexpr int E = 8 * D / kConsumerThreads;
    merge_heads<D, false>(p, recs, kConsumerWarps, R::SIZE, s, hg, scratch);
    const float* wk = scratch + kMaxSplits * 40;
    const int e0 = threadIdx.x * E, head = e0 / D;
    float acc[E];
#pragma unroll
    for (int x = 0; x < E; ++x) acc[x] = 0.f;
#pragma unroll
    for (int k = 0; k < kConsumerWarps; ++k) merge_accumulate<D>(acc, recs + k * R::SIZE, wk[k * 8 + head], e0);
    merge_emit<D>(p, acc, s, hg, scratch);
}

// the split records of one stream in the workspace (run by the stream's last
// CTA): scalars by loads, o vectors through bulk copies of a few records at a
// time into two shared-memory buffers (mbar[0], mbar[1]) behind the scratch
template <int D>
__device__ __forceinline__ void merge_splits(const DecodeParams& p, const float* base, int n, int s,
                                            int hg, uint8_t* smem, uint64_t* mbar,
                                            float* grec = nullptr) {
    using R = RecLayout<D>;
    constexpr int E = 8 * D / kConsumerThreads;
    constexpr int RB = R::SIZE * 4;                      // record bytes (multiple of 16)
    constexpr int BUF0 = (kMergeScratch + 127) & ~127;
    // records per bulk copy: two buffers in the ring behind the scratch
    constexpr int kMergeBatch = (kStages * Ring<D>::SLOT - BUF0) / (2 * RB);
    static_assert(RB % 16 == 0 && kMergeBatch >= 2, "merge buffers must fit in the ring");
    float* scratch = reinterpret_cast<float*>(smem);
    if (n <= kDirectMerge) {
        // few records: every o-vector load is issued before the scalar pass,
        // so both share one round of latency (no bulk-copy round trip)
        constexpr int E4 = 8 * D / kConsumerThreads / 4;
        const int e0 = threadIdx.x * (8 * D / kConsumerThreads);
        float4 v[kDirectMerge][E4];
#pragma unroll
        for (int u = 0; u < kDirectMerge; ++u)
#pragma unroll
            for (int j = 0; j < E4; ++j)
                if (u < n) v[u][j] = ld4<true>(base + u * R::SIZE + R::O + e0 + 4 * j);
        merge_heads<D, true>(p, base, n, R::SIZE, s, hg, scratch, grec);
        const float* wk = scratch + kMaxSplits * 40;
        const int head = e0 / D;
        float acc[E4 * 4];
#pragma unroll
        for (int x = 0; x < E4 * 4; ++x) acc[x] = 0.f;
#pragma unroll
        for (int u = 0; u < kDirectMerge; ++u) {
            if (u < n) {
                const float wgt = wk[u * 8 + head];
#pragma unroll
                for (int j = 0; j < E4; ++j) {
                    acc[4 * j + 0] = fmaf(wgt, v[u][j].x, acc[4 * j + 0]);
                    acc[4 * j + 1] = fmaf(wgt, v[u][j].y, acc[4 * j + 1]);
                    acc[4 * j + 2] = fmaf(wgt, v[u][j].z, acc[4 * j + 2]);
                    acc[4 * j + 3] = fmaf(wgt, v[u][j].w, acc[4 * j + 3]);
                }
            }
        }
        merge_emit<D>(p, acc, s, hg, scratch, grec);
        return;
    }
    {
        // few active q heads in this head group (G < 8): only their nh x D
        // outputs are merged.  They form CH float4 chunks; the threads split
        // into RGN groups of CH, group gi taking records gi, gi + RGN, ...,
        // every load issued before the scalar pass (one round of latency,
        // no bulk-copy round trips), then the groups' sums are reduced
        // through shared memory behind the scratch.
        const int nh = min(kHeadsPerTile, p.G - hg * kHeadsPerTile);
        const int CH = nh * D / 4;
        const int RGN = CH <= kConsumerThreads ? kConsumerThreads / CH : 0;
        if (grec == nullptr && RGN > 0 && n <= kNarrowLoads * RGN) {
            const int c = threadIdx.x % CH, gi = threadIdx.x / CH;
            const bool act = gi < RGN;
            float4 v[kNarrowLoads];
#pragma unroll
            for (int j = 0; j < kNarrowLoads; ++j) {
                const int u = gi + j * RGN;
                if (act && u < n) v[j] = ld4<true>(base + u * R::SIZE + R::O + 4 * c);
            }
            merge_heads<D, true>(p, base, n, R::SIZE, s, hg, scratch);
            const float* wk = scratch + kMaxSplits * 40;
            const int head = (4 * c) / D;
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < kNarrowLoads; ++j) {
                const int u = gi + j * RGN;
                if (act && u < n) {
                    const float wgt = wk[u * 8 + head];
                    a.x = fmaf(wgt, v[j].x, a.x);
                    a.y = fmaf(wgt, v[j].y, a.y);
                    a.z = fmaf(wgt, v[j].z, a.z);
                    a.w = fmaf(wgt, v[j].w, a.w);
                }
            }
            float4* red = reinterpret_cast<float4*>(smem + BUF0);   // [RGN][CH]
            if (act) red[gi * CH + c] = a;
            named_sync(1, kConsumerThreads);
            const int e0 = threadIdx.x * E;
            float acc[E];
#pragma unroll
            for (int x = 0; x < E; ++x) acc[x] = 0.f;
            if (e0 < nh * D) {
#pragma unroll
                for (int j = 0; j < E / 4; ++j) {
                    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int g = 0; g < RGN; ++g) {
                        const float4 q = red[g * CH + e0 / 4 + j];
                        t.x += q.x; t.y += q.y; t.z += q.z; t.w += q.w;
                    }
                    acc[4 * j] = t.x; acc[4 * j + 1] = t.y; acc[4 * j + 2] = t.z; acc[4 * j + 3] = t.w;
                }
            }
            merge_emit<D>(p, acc, s, hg, scratch);
            return;
        }
    }
    const int nb = (n + kMergeBatch - 1) / kMergeBatch;
    auto issue = [&](int bi) {
        const int cnt = min(kMergeBatch, n - bi * kMergeBatch);
        uint8_t* dst = smem + BUF0 + (bi & 1) * kMergeBatch * RB;
        bulk_g2s(dst, base + (int64_t)bi * kMergeBatch * R::SIZE, (uint32_t)(cnt * RB), mbar + (bi & 1));
        mbar_arrive_expect_tx(mbar + (bi & 1), (uint32_t)(cnt * RB));
    };
    if (threadIdx.x == 0) {
        // records written by other CTAs (generic proxy, ordered by the ticket)
        // and this CTA's earlier shared-memory use, before async-proxy copies
        asm volatile("fence.proxy.async.global;\n" ::: "memory");
        fence_proxy_async();
        for (int bi = 0; bi < min(nb, 2); ++bi) issue(bi);
    }
    merge_heads<D, true>(p, base, n, R::SIZE, s, hg, scratch, grec);
    const float* wk = scratch + kMaxSplits * 40;
    const int e0 = threadIdx.x * E, head = e0 / D;
    float acc[E];
#pragma unroll
    for (int x = 0; x < E; ++x) acc[x] = 0.f;
    for (int bi = 0; bi < nb; ++bi) {
        if (!mbar_wait(mbar + (bi & 1), (bi >> 1) & 1)) atomicExch(p.status, FKV_ERR_TIMEOUT);
        const float* buf = reinterpret_cast<const float*>(smem + BUF0 + (bi & 1) * kMergeBatch * RB);
        const int cnt = min(kMergeBatch, n - bi * kMergeBatch);
        for (int u = 0; u < cnt; ++u)
            merge_accumulate<D>(acc, buf + u * R::SIZE, wk[(bi * kMergeBatch + u) * 8 + head], e0);
        named_sync(1, kConsumerThreads);   // buffer (bi & 1) is free again
        if (threadIdx.x == 0 && bi + 2 < nb) issue(bi + 2);
    }
    merge_emit<D>(p, acc, s, hg, scratch, grec);
}

// Cluster mode: merge the csize CTA records of one cluster (each in its CTA's
// shared memory at `crec`) through distributed shared memory.  The 8 x D
// outputs are spread over the cluster's consumer threads; every thread loads
// the (m, l, o) of its element from each rank in one round, then emits the
// output (or the sequence-split record, or, with several groups per stream,
// the cluster's record in the workspace).  Rank 0 merges the spike trackers.
constexpr int kMaxCluster = 16;

template <int D>
__device__ __forceinline__ void cluster_merge(const DecodeParams& p, int s, int hg, int grp,
                                              int crank, const float* crec) {
    using R = RecLayout<D>;
    const int C = p.csize;
    const int b = s / p.Hk, h = s % p.Hk;
    uint32_t base[kMaxCluster];
#pragma unroll
    for (int k = 0; k < kMaxCluster; ++k) base[k] = k < C ? peer_smem(crec, (uint32_t)k) : 0u;
    float* grec = p.groups > 1 ? p.ws + (((int64_t)s * p.HG + hg) * p.groups + grp) * R::SIZE : nullptr;
    for (int e = crank * kConsumerThreads + (int)threadIdx.x; e < kHeadsPerTile * D;
         e += C * kConsumerThreads) {
        const int head = e / D, d = e % D;
        float mv[kMaxCluster], lv[kMaxCluster], ov[kMaxCluster];
#pragma unroll
        for (int k = 0; k < kMaxCluster; ++k) {
            if (k < C) {
                mv[k] = ld_peer_f32(base[k] + 4u * (R::M + head));
                lv[k] = ld_peer_f32(base[k] + 4u * (R::L + head));
                ov[k] = ld_peer_f32(base[k] + 4u * (R::O + e));
            }
        }
        float M = -INFINITY;
#pragma unroll
        for (int k = 0; k < kMaxCluster; ++k)
            if (k < C) M = fmaxf(M, mv[k]);
        float L = 0.f, acc = 0.f;
#pragma unroll
        for (int k = 0; k < kMaxCluster; ++k) {
            if (k < C) {
                const float wgt = mv[k] == -INFINITY ? 0.f : exp2f((mv[k] - M) * kLog2e);
                L = fmaf(wgt, lv[k], L);
                acc = fmaf(wgt, ov[k], acc);
            }
        }
        const int g = hg * kHeadsPerTile + head;
        if (grec != nullptr) {
            grec[R::O + e] = acc;
            if (d == 0) {
                grec[R::M + head] = M;
                grec[R::L + head] = L;
            }
        } else if (g < p.G) {
            const int64_t bh = (int64_t)b * p.Hq + (int64_t)h * p.G + g;
            if (p.part != nullptr) {
                p.part[bh * (D + 4) + 4 + d] = acc;
                if (d == 0) {
                    p.part[bh * (D + 4)] = M;
                    p.part[bh * (D + 4) + 1] = L;
                }
            } else {
                p.out[bh * D + d] = __half_as_ushort(__float2half_rn(L > 0.f ? acc / L : 0.f));
            }
        }
    }
    if (crank == 0 && threadIdx.x < kHeadsPerTile) {
        const int head = threadIdx.x;
        float mn = INFINITY, mf = -INFINITY;
        int af = -1;
        for (int k = 0; k < C; ++k) {
            const uint32_t bk = peer_smem(crec, (uint32_t)k);
            mn = fminf(mn, ld_peer_f32(bk + 4u * (R::MN + head)));
            argmax_merge(mf, af, ld_peer_f32(bk + 4u * (R::MF + head)), ld_peer_s32(bk + 4u * (R::AF + head)));
        }
        const int g = hg * kHeadsPerTile + head;
        if (grec != nullptr) {
            grec[R::MN + head] = mn;
            grec[R::MF + head] = mf;
            grec[R::AF + head] = __int_as_float(af);
        } else if (g < p.G) {
            const int64_t bh = (int64_t)b * p.Hq + (int64_t)h * p.G + g;
            if (p.part != nullptr) {
                p.part[bh * (D + 4) + 2] = mn;
                p.part[bh * (D + 4) + 3] = mf;
                p.part_arg[bh] = af >= 0 ? af + p.far_offset : -1;
            } else {
                p.flags[bh] = (mf > mn + p.margin) ? 1 : 0;
                p.tokens[bh] = af;
            }
        }
    }
}

// NH = 0: far-tier q.K on mma.sync after converting the codes; NH = 4 or 8:
// far-tier q.K on tcgen05 (NH q heads per CTA, D = 128, E4M3 K; maps.far_k
// is used only then).
// CL: cluster mode.  The CTAs of one cluster share the stage range of one
// (stream, head group, group of the stream's cost ranges): the first kStages
// stages are dealt round robin, the rest claimed one at a time through a
// counter in the shared memory of cluster rank 0, so CTAs that run faster
// take more stages; the CTA records are then merged through distributed
// shared memory instead of global records and a ticket.
// RT: the progress waits take the caller's iteration limit (p.wait_limit) and
// the test hook p.test_stall is honoured; without RT both are compile-time
// (the fixed limit, no hook), which keeps the hot loop's registers down.
template <int D, int VG, int NH = 0, bool CL = false, bool RT = false>
__global__ void __maxnreg__((NH > 0 || CL || VG == kTurbo) ? 128 : 136)
    decode_fp8_kernel(const DecodeParams p, const __grid_constant__ TMaps maps) {
    using R = RecLayout<D>;
    using RG = Ring<D, VG>;
    using UL = UmLayout<D, VG>;
    constexpr bool UM = NH > 0;
    static_assert(!UM || (D == 128 && VG != kTurbo), "tensor-core far path: fp8 K, D = 128");
    static_assert(!(UM && CL), "cluster mode runs on the mma.sync far path");
    const uint32_t wlim = RT ? p.wait_limit : kWaitLimit;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // 1024-byte aligned base: the swizzled TMA boxes and UMMA operands
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + RG::BAROFF);
    uint4* qs = reinterpret_cast<uint4*>(smem + RG::QOFF);
    uint64_t* empty = full + kStages;
    __shared__ int sh_last;
    const int hg = blockIdx.y, s = blockIdx.z;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    // cluster mode: this CTA's rank in its cluster and the cluster's group;
    // the group plays the role of the split in the cost-range cut below
    const int crank = CL ? (int)cluster_rank() : 0;
    const int split = CL ? (int)blockIdx.x / p.csize : (int)blockIdx.x;
    const int nsplit = CL ? p.groups : p.splits;
    int* hdr = reinterpret_cast<int*>(smem + RG::HDR);
    volatile int* issued_c = reinterpret_cast<volatile int*>(smem + RG::ISSUED);
    volatile int* pdone = reinterpret_cast<volatile int*>(smem + RG::PDONE);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, kConsumerWarps);
        }
        mbar_init(reinterpret_cast<uint64_t*>(smem + RG::MERGEBAR), 1);
        mbar_init(reinterpret_cast<uint64_t*>(smem + RG::MERGEBAR) + 1, 1);
        mbar_init(reinterpret_cast<uint64_t*>(smem + RG::STALLBAR), 1);
        if constexpr (CL) {
            // rank 0's counter: the first kStages * csize stages are dealt round robin
            *reinterpret_cast<uint32_t*>(smem + RG::COUNTER) = (uint32_t)(kStages * p.csize);
            *issued_c = 0;
            *pdone = 0;
        }
        if constexpr (UM) {
            for (int i = 0; i < kStages; ++i) mbar_init(reinterpret_cast<uint64_t*>(smem + UL::MMAB) + i, 1);
            mbar_init(reinterpret_cast<uint64_t*>(smem + UL::QREADY), 3);   // TMEM + 2 piece warps
            mbar_init(reinterpret_cast<uint64_t*>(smem + UL::DRAIN), 1);
        }
        fence_mbar_init();
    }
    // Launched with programmatic stream serialization, this grid may start
    // while the previous kernel of the stream is still running (the set-up
    // above overlaps its tail): every global read waits here for it to
    // complete and its writes to be visible -- except on the TurboQuant path,
    // whose predecessor is the q-projection kernel, read by warp 0 only after
    // its own wait below.  Without a programmatic predecessor this returns
    // at once.
    if constexpr (VG != kTurbo || CL) asm volatile("griddepcontrol.wait;\n" ::: "memory");
    // segments of this split's share of the stream's work: the stream's
    // tokens [near valid | far | decode], weighted near_w / far_w / near_w
    // cost units, are cut into p.splits equal cost ranges (the near tier
    // counts only its near_valid rows, read here)
    const int nv = min(max(__ldg(p.near_valid + s), 0), p.Np);
    const int64_t nw = p.near_w, fw = p.far_w;
    const int64_t cost_near = nw * nv, cost_nf = cost_near + fw * p.F,
                  total_cost = cost_nf + nw * p.n_dec;
    auto to_tok = [&](int64_t cu) -> int {
        if (cu <= cost_near) return (int)(cu / nw);
        if (cu <= cost_nf) return nv + (int)((cu - cost_near) / fw);
        return nv + p.F + (int)((cu - cost_nf) / nw);
    };
    const int64_t chunk = (total_cost + nsplit - 1) / nsplit;
    const int t0 = to_tok(min((int64_t)split * chunk, total_cost));
    const int t1 = to_tok(min((int64_t)(split + 1) * chunk, total_cost));
    Segs sg;
    sg.a[0] = t0;                    sg.e[0] = min(t1, nv);
    sg.a[1] = max(t0, nv) - nv;      sg.e[1] = min(t1, nv + p.F) - nv;
    sg.a[2] = max(t0, nv + p.F) - nv - p.F;
    sg.e[2] = min(t1, nv + p.F + p.n_dec) - nv - p.F;
    sg.n[0] = sg.e[0] > sg.a[0] ? (sg.e[0] - sg.a[0] + RG::NEAR_TOK - 1) / RG::NEAR_TOK : 0;
    sg.n[1] = sg.e[1] > sg.a[1] ? (sg.e[1] - sg.a[1] + RG::FAR_TOK - 1) / RG::FAR_TOK : 0;
    sg.n[2] = sg.e[2] > sg.a[2] ? (sg.e[2] - sg.a[2] + RG::NEAR_TOK - 1) / RG::NEAR_TOK : 0;
    const int nstage = sg.n[0] + sg.n[1] + sg.n[2];
    __syncthreads();

    if (w == kConsumerWarps) {
        // ---------------- producer warp: one elected lane issues bulk copies
        [[maybe_unused]] int j = 0;          // cluster mode: stages put into this CTA's ring
        [[maybe_unused]] bool done = false;  // cluster mode: the sentinel header is out
        {
            const uint8_t* fk = p.far_k + (int64_t)s * p.F * D;
            const uint8_t* fv = p.far_v + (int64_t)s * p.F * (D / 2);
            // copies of stage k into slot k % kStages, completing on full[slot]
            auto issue = [&](int k, int slot) {
                int seg, start, cnt;
                stage_at<D>(sg, k, seg, start, cnt);
                uint8_t* dst = smem + slot * RG::SLOT;
                const uint8_t *ks, *vs;
                uint32_t kb, vb;
                if (seg == 1 && UM) {
                    ks = nullptr;                                          // tensor-map copy below
                    vs = fv + (int64_t)start * (D / 2);
                    kb = RG::FAR_TOK * D;                                  // whole box, rows past
                    vb = cnt * (D / 2);                                    // the stream are unused
                } else if (seg == 1 && VG == kTurbo) {
                    ks = p.far_k + ((int64_t)s * p.F + start) * (D / 4);   // 2-bit key codes
                    vs = p.far_v + ((int64_t)s * p.F + start) * (D / 4);   // 2-bit value codes
                    kb = vb = cnt * (D / 4);
                } else if (seg == 1) {
                    ks = fk + (int64_t)start * D;
                    vs = fv + (int64_t)start * (D / 2);
                    kb = cnt * D;
                    vb = cnt * (D / 2);
                } else {
                    ks = vs = nullptr;                                     // tensor-map copies below
                    kb = vb = RG::NEAR_TOK * D * 2;                        // whole boxes
                }
                if (seg != 1) {
                    const CUtensorMap* mk = seg == 0 ? &maps.near_k : &maps.dec_k;
                    const CUtensorMap* mv = seg == 0 ? &maps.near_v : &maps.dec_v;
                    const int row = (int)((int64_t)s * (seg == 0 ? p.Np : p.dec_stride) + start);
#pragma unroll
                    for (int hh = 0; hh < 2 * D / 128; ++hh) {
                        tma_load_2d(dst + hh * kHalfBox, mk, 64 * hh, row, full + slot);
                        tma_load_2d(dst + RG::VOFF + hh * kHalfBox, mv, 64 * hh, row, full + slot);
                    }
                } else {
                    if (UM) tma_load_2d(dst, &maps.far_k, 0, (int)((int64_t)s * p.F + start), full + slot);
                    else bulk_g2s(dst, ks, kb, full + slot);
                    bulk_g2s(dst + RG::VOFF, vs, vb, full + slot);
                }
                uint32_t tx = kb + vb;
                if (seg == 1) {
                    const int64_t row0 = (int64_t)s * p.F + start, nrows = (int64_t)p.B * p.Hk * p.F;
                    uint8_t* sd = dst + RG::SZOFF;
                    if constexpr (VG == kTurbo) {
                        const int64_t vsb = 2 * (D / 32);
                        tx += copy_covering(sd, (const uint8_t*)p.k_norm, nrows * 2, row0 * 2,
                                            (row0 + cnt) * 2, full + slot);
                        tx += copy_covering(sd + RG::RB0, (const uint8_t*)p.k_gamma, nrows * 2,
                                            row0 * 2, (row0 + cnt) * 2, full + slot);
                        tx += copy_covering(sd + 2 * RG::RB0, (const uint8_t*)p.v_scale, nrows * vsb,
                                            row0 * vsb, (row0 + cnt) * vsb, full + slot);
                        tx += copy_covering(sd + 2 * RG::RB0 + RG::RB2, p.k_signs, nrows * (D / 8),
                                            row0 * (D / 8), (row0 + cnt) * (D / 8), full + slot);
                    } else {
                        const int64_t eb = 2 * RG::SEL;
                        tx += copy_covering(sd, (const uint8_t*)p.v_scale, nrows * eb, row0 * eb,
                                            (row0 + cnt) * eb, full + slot);
                        tx += copy_covering(sd + RG::RB0, (const uint8_t*)p.v_zero, nrows * eb,
                                            row0 * eb, (row0 + cnt) * eb, full + slot);
                    }
                }
                mbar_arrive_expect_tx(full + slot, tx);
            };
            if (lane != 0) {
                // only the elected lane issues
            } else if constexpr (CL) {
                // first kStages stages dealt round robin (no wait: the slots
                // are free), then one claim per freed slot from rank 0's
                // counter (below); a claim past the end becomes a sentinel
                for (; j < kStages; ++j) {
                    const int k = crank + j * p.csize;
                    hdr[j] = k < nstage ? k : -1;
                    if (k >= nstage) {
                        mbar_arrive(full + j);
                        ++j;
                        done = true;
                        break;
                    }
                    issue(k, j);
                }
                *issued_c = j;
            } else if constexpr (!UM) {
                for (int k = 0; k < nstage; ++k) {
                    if (k >= kStages &&
                        !mbar_wait(empty + k % kStages, ((k / kStages) - 1) & 1, wlim)) {
                        atomicExch(p.status, FKV_ERR_TIMEOUT);
                        break;
                    }
                    issue(k, k % kStages);
                }
            } else {
                // Two event streams polled without blocking: refill a slot as
                // soon as the consumers release it (copies run kStages ahead,
                // as on the mma.sync path), and issue a far stage's MMA as
                // soon as its data lands.  Idle polls back off with a short
                // sleep; a long run of idle polls is a timeout.
                uint64_t* mmab = reinterpret_cast<uint64_t*>(smem + UL::MMAB);
                uint64_t* qready = reinterpret_cast<uint64_t*>(smem + UL::QREADY);
                bool ok = true, any_mma = false, have_t = false;
                uint32_t tbase = 0, idle = 0;
                int kc = 0, km = 0;
                while (km < nstage) {
                    bool prog = false;
                    if (km < kc && mbar_test(full + km % kStages, (km / kStages) & 1)) {
                        const int slot = km % kStages;
                        int seg, start, cnt;
                        stage_at<D>(sg, km, seg, start, cnt);
                        if (seg != 1) {
                            mbar_arrive(mmab + slot);   // keeps the barrier's phase = stage use
                            ++km;
                            prog = true;
                        } else if (have_t || mbar_test(qready, 0)) {
                            if (!have_t) {
                                tc_fence_after();
                                tbase = *reinterpret_cast<volatile uint32_t*>(smem + UL::TADDR);
                                have_t = true;
                            }
                            tc_fence_after();
                            const uint32_t a0 = smem_u32(smem + slot * RG::SLOT);
                            const uint32_t b0 = smem_u32(smem + UL::QB);
                            constexpr uint32_t idesc = f8_idesc(128, kQPieces * NH);
#pragma unroll
                            for (int j = 0; j < D / 32; ++j)
                                umma_f8(tbase + slot * 32, sw128_kmajor_desc(a0 + 32 * j),
                                        sw128_kmajor_desc(b0 + 32 * j), idesc, j > 0);
                            umma_commit(mmab + slot);
                            any_mma = true;
                            ++km;
                            prog = true;
                        }
                    }
                    if (kc < nstage &&
                        (kc < kStages || mbar_test(empty + kc % kStages, ((kc / kStages) - 1) & 1))) {
                        issue(kc, kc % kStages);
                        ++kc;
                        prog = true;
                    }
                    if (prog) {
                        idle = 0;
                    } else if (++idle > wlim) {
                        ok = false;
                        break;
                    } else {
                        __nanosleep(32);
                    }
                }
                if (!ok) atomicExch(p.status, FKV_ERR_TIMEOUT);
                // drain barrier: completes when every MMA issued above has
                // finished (the TMEM owner waits for it before freeing TMEM)
                uint64_t* drain = reinterpret_cast<uint64_t*>(smem + UL::DRAIN);
                if (any_mma) umma_commit(drain);
                else mbar_arrive(drain);
            }
            if constexpr (CL) {
                __syncwarp();
                cluster_arrive();   // start barrier: rank 0's counter is set, every CTA runs
                cluster_wait();
                if (lane == 0) {
                    // each claim is made one stage ahead, so the round trip to
                    // rank 0 overlaps the wait for the next free slot
                    const uint32_t ctr = peer_smem(smem + RG::COUNTER, 0);
                    int k_next = done ? nstage : (int)atom_add_peer(ctr, 1u);
                    while (!done) {
                        const int slot = j % kStages;
                        if (!mbar_wait(empty + slot, ((j / kStages) - 1) & 1, wlim)) {
                            atomicExch(p.status, FKV_ERR_TIMEOUT);
                            break;
                        }
                        const int k = k_next;
                        if (k < nstage) k_next = (int)atom_add_peer(ctr, 1u);
                        hdr[slot] = k < nstage ? k : -1;
                        if (k < nstage) {
                            issue(k, slot);
                        } else {
                            mbar_arrive(full + slot);
                            done = true;
                        }
                        ++j;
                        *issued_c = j;
                    }
                    __threadfence_block();
                    *pdone = 1;
                }
                __syncwarp();
                cluster_arrive();   // end barrier 1: the CTA records are in shared memory
                cluster_wait();
                cluster_arrive();   // end barrier 2: the merge has read them
                cluster_wait();
            }
        }
        asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
        return;
    }

    // ---------------- consumer warps
    uint4* qr = qs + RG::QFRAG / 16;
    uint4* qk = qr + RG::QFRAG / 16;
    float* tsum = reinterpret_cast<float*>(smem + RG::TSUM);
    // start-up work in parallel: warp 0 the mma.sync q fragments (+ turbo
    // fragments); on the tensor-core path warp 1 allocates TMEM (and frees it
    // at the end) while warps 2 and 3 build the q-piece B operand
    if (w == 0) {
        build_q_frags<D>(p, s, hg, lane, qs);
        if constexpr (VG == kTurbo && !CL) {
            // q Pi^T / q S^T come from turbo_qproj_kernel, which may still be
            // running (programmatic dependent launch): wait for it here only
            asm volatile("griddepcontrol.wait;\n" ::: "memory");
            build_turbo_frags<D>(p, s, hg, lane, qr, qk, tsum);
        }
    }
    if constexpr (CL) {
        float* qpj = reinterpret_cast<float*>(smem + RG::QPJ);
        if constexpr (VG == kTurbo) turbo_qproj_slice<D>(p, s, hg, crank, qpj);
        __syncwarp();
        cluster_arrive();   // start barrier (with the producer warps of the cluster)
        cluster_wait();
        if constexpr (VG == kTurbo) {
            turbo_qproj_gather<D>(p, crank, qpj);
            named_sync(1, kConsumerThreads);
            if (w == 0) build_turbo_frags<D>(p, s, hg, lane, qr, qk, tsum, qpj);
        }
    }
    if constexpr (UM) {
        if (w >= 1) {
            if (w == 1) tmem_alloc(reinterpret_cast<uint32_t*>(smem + UL::TADDR), UL::TMEM_COLS);
            else build_q_pieces<D, NH>(p, s, hg, w - 2, lane, smem + UL::QB,
                                       reinterpret_cast<float*>(smem + UL::ESC));
            fence_proxy_async();   // B operand -> tensor-core reads
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(reinterpret_cast<uint64_t*>(smem + UL::QREADY));
        }
    }
    named_sync(1, kConsumerThreads);
    uint32_t tbase = 0;
    float escale = 1.f;
    if constexpr (UM) {
        tc_fence_after();
        tbase = *reinterpret_cast<volatile uint32_t*>(smem + UL::TADDR);
        escale = *reinterpret_cast<volatile float*>(smem + UL::ESC);
    }
    float cf[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float sum_r = 0.f, sum_k = 0.f;
    if constexpr (VG == kTurbo) {
        const float c0 = __ldg(p.centroids), c1 = __ldg(p.centroids + 1);
        const float c2 = __ldg(p.centroids + 2), c3 = __ldg(p.centroids + 3);
        // c[code] = c0 + (c1 - c0) b0 + (c2 - c0) b1 + ((c3 - c2) - (c1 - c0)) b0 b1
        // for the code's bits b0 (low) and b1; the b0 b1 term vanishes for the
        // symmetric Lloyd-Max centroids, and its tensor-core product with it
        cf[0] = c0; cf[1] = c1 - c0; cf[2] = c2 - c0; cf[3] = (c3 - c2) - (c1 - c0);
        cf[4] = p.qjl_coef / (float)D;
        cf[5] = p.qscale;
        sum_r = tsum[lane >> 2];
        sum_k = tsum[8 + (lane >> 2)];
    }
    WarpState<D> st;
    st.init();
    const int64_t srow0 = (int64_t)s * p.F;
    int failed_at = -1;
    if (RT && p.test_stall) {
        // test hook: a wait that nothing satisfies, so the timeout path runs
        // (error status, bounded drain of the copies in flight, normal exit)
        // without any fault
        if (!mbar_wait(reinterpret_cast<uint64_t*>(smem + RG::STALLBAR), 0, wlim)) {
            atomicExch(p.status, FKV_ERR_TIMEOUT);
            failed_at = 0;
        }
    }
    // stage sequence of this CTA's ring: its own stages 0..nstage-1, or in
    // cluster mode the stages named by the slot headers up to a sentinel
    const int nloop = failed_at >= 0 ? 0 : CL ? INT_MAX : nstage;
    for (int jj = 0; jj < nloop; ++jj) {
        const int slot = jj % kStages;
        int k = jj;
        int seg, start, cnt;
        if constexpr (!CL) stage_at<D>(sg, k, seg, start, cnt);
        // (outside cluster mode the consumers' data waits keep the fixed
        // limit; the stall test never reaches them)
        if (!mbar_wait(full + slot, (jj / kStages) & 1, wlim)) {
            atomicExch(p.status, FKV_ERR_TIMEOUT);
            failed_at = jj;
            break;
        }
        if constexpr (CL) {
            k = *reinterpret_cast<volatile int*>(hdr + slot);
            if (k < 0) break;   // sentinel: the cluster's stages are all taken
            stage_at<D>(sg, k, seg, start, cnt);
        }
        uint8_t* kbuf = smem + slot * RG::SLOT;
        const uint8_t* vbuf = kbuf + RG::VOFF;
        const int ntile = (cnt + kTile - 1) / kTile;
        if (UM && seg == 1) {
            uint64_t* mmab = reinterpret_cast<uint64_t*>(smem + UL::MMAB) + slot;
            const uint32_t par = (k / kStages) & 1;
            bool ok = true;
            const int64_t row0 = srow0 + start;
            constexpr int eb = 2 * RG::SEL;
            const uint8_t* sd = kbuf + RG::SZOFF;
            const uint16_t* sc = reinterpret_cast<const uint16_t*>(sd + ((row0 * eb) & 15));
            const uint16_t* ze = reinterpret_cast<const uint16_t*>(sd + RG::RB0 + ((row0 * eb) & 15));
            const uint32_t ta = tbase + ((uint32_t)(32 * w) << 16) + (uint32_t)(slot * 32);
            if constexpr (UM) {
                if (32 * w + 16 < cnt) {
                    const int u0[2] = {32 * w, 32 * w + 16};
                    uint32_t sz[2][4];
                    load_sz<D, VG>(sc, ze, u0[0], cnt, lane, sz[0]);
                    load_sz<D, VG>(sc, ze, u0[1], cnt, lane, sz[1]);
                    ok = far_tiles_um<D, VG, 2, NH>(kbuf, vbuf, u0, cnt, start, lane, w, ta, escale, mmab,
                                                    par, wlim, sz, st);
                } else if (32 * w < cnt) {
                    const int u0[1] = {32 * w};
                    uint32_t sz[1][4];
                    load_sz<D, VG>(sc, ze, u0[0], cnt, lane, sz[0]);
                    ok = far_tiles_um<D, VG, 1, NH>(kbuf, vbuf, u0, cnt, start, lane, w, ta, escale, mmab,
                                                    par, wlim, sz, st);
                }
            }
            if (!ok) {
                atomicExch(p.status, FKV_ERR_TIMEOUT);
                failed_at = k;
                break;
            }
            tc_fence_before();    // TMEM reads ordered before the slot release
            fence_proxy_async();  // transpose writes ordered before the slot's next TMA fill
        } else if (seg == 1) {
            // stage scalars: covering copies start at the 16-byte boundary below
            const int64_t row0 = srow0 + start;
            const uint8_t* sd = kbuf + RG::SZOFF;
            if constexpr (VG == kTurbo) {
                const uint16_t* nm = reinterpret_cast<const uint16_t*>(sd + ((row0 * 2) & 15));
                const uint16_t* gm = reinterpret_cast<const uint16_t*>(sd + RG::RB0 + ((row0 * 2) & 15));
                const uint16_t* vsp = reinterpret_cast<const uint16_t*>(
                    sd + 2 * RG::RB0 + ((row0 * 2 * (D / 32)) & 15));
                const uint8_t* sgn = sd + 2 * RG::RB0 + RG::RB2 + ((row0 * (D / 8)) & 15);
#pragma unroll
                for (int x = 0; x < 2; ++x) {
                    const int i = w + 4 * x;
                    if (i < ntile) {
                        uint32_t ng[4], vs2[2];
                        load_turbo_sz<D>(nm, gm, vsp, i * kTile, cnt, lane, ng, vs2);
                        turbo_tile<D, CL>(sgn, kbuf, vbuf, i * kTile, cnt, srow0, start, lane, qr, qk,
                                      cf, sum_r, sum_k, ng, vs2, st);
                    }
                }
            } else {
                constexpr int eb = 2 * RG::SEL;
                const uint16_t* sc = reinterpret_cast<const uint16_t*>(sd + ((row0 * eb) & 15));
                const uint16_t* ze = reinterpret_cast<const uint16_t*>(sd + RG::RB0 + ((row0 * eb) & 15));
                if (w + 4 < ntile) {
                    const int u0[2] = {w * kTile, (w + 4) * kTile};
                    uint32_t sz[2][4];
                    load_sz<D, VG>(sc, ze, u0[0], cnt, lane, sz[0]);
                    load_sz<D, VG>(sc, ze, u0[1], cnt, lane, sz[1]);
                    far_tiles<D, VG, 2, CL>(kbuf, vbuf, u0, cnt, start, lane, qs, sz, st);
                } else if (w < ntile) {
                    const int u0[1] = {w * kTile};
                    uint32_t sz[1][4];
                    load_sz<D, VG>(sc, ze, u0[0], cnt, lane, sz[0]);
                    far_tiles<D, VG, 1, CL>(kbuf, vbuf, u0, cnt, start, lane, qs, sz, st);
                }
            }
        } else if (w < ntile) {
            fp16_tile<D>(kbuf, vbuf, w * kTile, cnt, lane, qs, st);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot);
    }
    // this CTA's tier stream is done: a programmatically launched next grid
    // may start its set-up (it waits for this grid's completion before any
    // global read) while the records are written and merged
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    if (failed_at >= 0) {
        // the producer runs at most kStages ahead of the consumers: wait
        // (bounded) for the copies it may still have in flight, then leave
        if constexpr (CL) {
            for (uint32_t i = 0; i < kWaitLimit && *pdone == 0; ++i) __nanosleep(64);
            const int iss = *issued_c;
            for (int jj = failed_at; jj < iss; ++jj)
                if (!mbar_wait(full + (jj % kStages), (jj / kStages) & 1)) break;
        } else {
            for (int k = failed_at; k < min(nstage, failed_at + kStages); ++k) {
                if (!mbar_wait(full + (k % kStages), (k / kStages) & 1)) break;
            }
        }
    }

    // ---- warp record -> shared memory (the ring is free once all consumers pass)
    const int r = lane >> 2, c = lane & 3;
    st.l = quad_sum(st.l);
    st.z = quad_sum(st.z);
    st.mn = quad_min(st.mn);
    quad_argmax(st.mf, st.af);
    const float z0 = __shfl_sync(0xffffffffu, st.z, (2 * c) * 4);
    const float z1 = __shfl_sync(0xffffffffu, st.z, (2 * c + 1) * 4);
    named_sync(1, kConsumerThreads);
    float* sh_rec = reinterpret_cast<float*>(smem);
    float* wr = sh_rec + w * R::SIZE;
    if (c == 0) {
        wr[R::M + r] = st.m;
        wr[R::L + r] = st.l;
        wr[R::MN + r] = st.mn;
        wr[R::MF + r] = st.mf;
        wr[R::AF + r] = __int_as_float(st.af);
    }
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
        const int d0 = r * (D / 8) + 2 * i;
        wr[R::O + (2 * c) * D + d0] = st.o[i][0] + z0;
        wr[R::O + (2 * c + 1) * D + d0] = st.o[i][1] + z1;
        wr[R::O + (2 * c) * D + d0 + 1] = st.o[i][2] + z0;
        wr[R::O + (2 * c + 1) * D + d0 + 1] = st.o[i][3] + z1;
    }
    named_sync(1, kConsumerThreads);
    if constexpr (UM) {
        if (w == 1) {
            // all consumer TMEM reads are done (barrier above); wait for the
            // producer's drain commit so no MMA is in flight, then free TMEM
            // (the allocating warp frees it)
            uint64_t* drain = reinterpret_cast<uint64_t*>(smem + UL::DRAIN);
            for (int i = 0; i < 4; ++i)
                if (mbar_wait(drain, 0)) break;
            tc_fence_after();
            tmem_dealloc(tbase, UL::TMEM_COLS);
        }
    }

    if (!CL && p.splits == 1) {
        merge_warps<D>(p, sh_rec, s, hg, sh_rec + kConsumerWarps * R::SIZE);
        return;
    }

    // ---- CTA record -> workspace (cluster mode: this CTA's shared memory),
    // then the last CTA of this stream merges
    float* cw = sh_rec + kConsumerWarps * R::SIZE;   // [warp][head] weights exp(m_w - M)
    float* gr = CL ? cw + kConsumerWarps * kHeadsPerTile
                   : p.ws + (((int64_t)s * p.HG + hg) * p.splits + split) * R::SIZE;
    if (threadIdx.x < kHeadsPerTile) {
        const int head = threadIdx.x;
        float M = -INFINITY, L = 0.f, mn = INFINITY, mf = -INFINITY;
        int af = -1;
#pragma unroll
        for (int k = 0; k < kConsumerWarps; ++k) M = fmaxf(M, sh_rec[k * R::SIZE + R::M + head]);
#pragma unroll
        for (int k = 0; k < kConsumerWarps; ++k) {
            const float* q = sh_rec + k * R::SIZE;
            const float wgt = (q[R::M + head] == -INFINITY) ? 0.f : exp2f((q[R::M + head] - M) * kLog2e);
            cw[k * kHeadsPerTile + head] = wgt;
            L = fmaf(wgt, q[R::L + head], L);
            mn = fminf(mn, q[R::MN + head]);
            argmax_merge(mf, af, q[R::MF + head], __float_as_int(q[R::AF + head]));
        }
        gr[R::M + head] = M;
        gr[R::L + head] = L;
        gr[R::MN + head] = mn;
        gr[R::MF + head] = mf;
        gr[R::AF + head] = __int_as_float(af);
    }
    named_sync(1, kConsumerThreads);
    for (int e = 4 * threadIdx.x; e < kHeadsPerTile * D; e += 4 * kConsumerThreads) {
        const int head = e / D;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < kConsumerWarps; ++k) {
            const float wgt = cw[k * kHeadsPerTile + head];
            const float4 o = *reinterpret_cast<const float4*>(sh_rec + k * R::SIZE + R::O + e);
            acc.x = fmaf(wgt, o.x, acc.x);
            acc.y = fmaf(wgt, o.y, acc.y);
            acc.z = fmaf(wgt, o.z, acc.z);
            acc.w = fmaf(wgt, o.w, acc.w);
        }
        *reinterpret_cast<float4*>(gr + R::O + e) = acc;
    }
    if constexpr (CL) {
        named_sync(1, kConsumerThreads);
        cluster_arrive();   // end barrier 1: every CTA record of the cluster is ready
        cluster_wait();
        cluster_merge<D>(p, s, hg, split, crank, gr);
        if (p.groups > 1) __threadfence();   // the cluster's record, before rank 0's ticket
        __syncwarp();
        cluster_arrive();   // end barrier 2: no peer reads this CTA's shared memory any more
        cluster_wait();
        if (p.groups == 1 || crank != 0) return;
        named_sync(1, kConsumerThreads);
        if (threadIdx.x == 0) {
            int* tk = p.tickets + ((int64_t)s * p.HG + hg);
            const int old = atomicAdd(tk, 1);
            sh_last = (old == p.groups - 1);
            if (sh_last) *tk = 0;
        }
        named_sync(1, kConsumerThreads);
        if (!sh_last) return;
        __threadfence();
        const float* gbase = p.ws + ((int64_t)s * p.HG + hg) * p.groups * R::SIZE;
        merge_splits<D>(p, gbase, p.groups, s, hg, smem,
                        reinterpret_cast<uint64_t*>(smem + RG::MERGEBAR));
        return;
    }
    __threadfence();
    named_sync(1, kConsumerThreads);
    const int64_t unit = (int64_t)s * p.HG + hg;
    uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + RG::MERGEBAR);
    if ((VG == kTurbo || UM) && p.splits > kDirectMerge) {
        // two-level merge (TurboQuant tier, whose small streams take many
        // splits, and the tensor-core q.K kernels, which stay within their
        // 128 registers with it; in the mma.sync fp8 kernels the extra code
        // cost the hot loop registers and c3 4 %): the last CTA of each group of kMergeGroup splits
        // merges them into a group record (one round of loads), the last
        // group merges the group records -- instead of one CTA streaming
        // every split record through shared memory
        const int ngrp = (p.splits + kMergeGroup - 1) / kMergeGroup;
        const int grp = split / kMergeGroup;
        const int gn = min(kMergeGroup, p.splits - grp * kMergeGroup);
        const int64_t units = (int64_t)gridDim.y * gridDim.z;
        if (threadIdx.x == 0) {
            int* tk = p.tickets + units + unit * ngrp + grp;
            const int old = atomicAdd(tk, 1);
            sh_last = (old == gn - 1);
            if (sh_last) *tk = 0;
        }
        named_sync(1, kConsumerThreads);
        if (!sh_last) return;
        __threadfence();
        float* grecs = p.ws + units * p.splits * R::SIZE + unit * ngrp * R::SIZE;
        merge_splits<D>(p, p.ws + (unit * p.splits + grp * kMergeGroup) * R::SIZE, gn, s, hg, smem, mbar,
                        grecs + grp * R::SIZE);
        __threadfence();
        named_sync(1, kConsumerThreads);
        if (threadIdx.x == 0) {
            int* tk = p.tickets + unit;
            const int old = atomicAdd(tk, 1);
            sh_last = (old == ngrp - 1);
            if (sh_last) *tk = 0;
        }
        named_sync(1, kConsumerThreads);
        if (!sh_last) return;
        __threadfence();
        merge_splits<D>(p, grecs, ngrp, s, hg, smem, mbar);
        return;
    }
    if (threadIdx.x == 0) {
        int* tk = p.tickets + unit;
        const int old = atomicAdd(tk, 1);
        sh_last = (old == p.splits - 1);
        if (sh_last) *tk = 0;   // every other CTA of this stream has arrived
    }
    named_sync(1, kConsumerThreads);
    if (!sh_last) return;
    __threadfence();
    const float* base = p.ws + unit * p.splits * R::SIZE;
    merge_splits<D>(p, base, p.splits, s, hg, smem, mbar);
}

// shard k's record n at parts + k * prs + n * (D + 4), its argmax at
// args + k * ars + n (prs / ars: element strides between the shards' blocks).
// With a gathered [records | argmax] layout the stride N * (D + 4) + N is
// usually not a multiple of 4 floats, so a record may be only 4-byte
// aligned: this kernel reads the records with scalar loads only.
template <int D>
__global__ void combine_kernel(int P, int N, const float* __restrict__ parts, int64_t prs,
                               const int32_t* __restrict__ args, int64_t ars, float margin,
                               uint16_t* __restrict__ out, int32_t* __restrict__ flags,
                               int32_t* __restrict__ tokens) {
    const int n = blockIdx.x;
    const int64_t rs = D + 4;
    float M = -INFINITY;
    for (int k = 0; k < P; ++k) M = fmaxf(M, parts[k * prs + n * rs]);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float L = 0.f, acc = 0.f;
        if (M != -INFINITY) {
            for (int k = 0; k < P; ++k) {
                const float* rec = parts + k * prs + n * rs;
                if (rec[0] == -INFINITY) continue;
                const float wgt = exp2f((rec[0] - M) * kLog2e);
                L = fmaf(wgt, rec[1], L);
                acc = fmaf(wgt, rec[4 + d], acc);
            }
        }
        out[(int64_t)n * D + d] = __half_as_ushort(__float2half_rn(L > 0.f ? acc / L : 0.f));
    }
    if (threadIdx.x == 0) {
        float mn = INFINITY, mf = -INFINITY;
        int af = -1;
        for (int k = 0; k < P; ++k) {
            const float* rec = parts + k * prs + n * rs;
            mn = fminf(mn, rec[2]);
            if (rec[3] > mf) {   // shard order: first shard with the strict max wins
                mf = rec[3];
                af = args[k * ars + n];
            }
        }
        flags[n] = (mf > mn + margin) ? 1 : 0;
        tokens[n] = af;
    }
}

int g_num_sms = 0;

int num_sms() {
    if (g_num_sms == 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return 148;
        if (cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            g_num_sms = 148;
    }
    return g_num_sms;
}

// Resident CTAs per SM of one decode kernel instantiation (queried once per
// device after opting it into its dynamic shared memory).
using KernelFn = void (*)(DecodeParams, TMaps);

int resident_ctas(KernelFn kern, int smem, int tmem_cols = 0) {
    static thread_local std::vector<std::pair<std::pair<int, const void*>, int>> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 2;
    for (auto& e : cache)
        if (e.first.first == dev && e.first.second == (const void*)kern) return e.second;
    int n = 2;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, smem) != cudaSuccess || n < 1)
        n = 2;
    if (tmem_cols > 0) {
        // the occupancy query answers 1 for kernels that allocate tensor
        // memory; bound residency by registers, shared memory, threads and
        // TMEM columns instead
        cudaFuncAttributes fa{};
        int sm_smem = 0, reserved = 0;
        if (cudaFuncGetAttributes(&fa, (const void*)kern) == cudaSuccess &&
            cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) == cudaSuccess) {
            // registers are allocated per warp in units of 8 per thread, from
            // the 16K-register file of the sub-partition the warp runs on
            const int warps = (kThreads + 31) / 32;
            const int regs_warp = ((fa.numRegs + 7) / 8) * 8 * 32;
            int by_regs = 0;
            while (((by_regs + 1) * warps + 3) / 4 * regs_warp <= 16384) ++by_regs;
            const int by_smem = sm_smem / std::max(1, smem + (int)fa.sharedSizeBytes + reserved);
            const int by_threads = 2048 / kThreads;
            const int by_tmem = 512 / tmem_cols;
            n = std::max(1, std::min(std::min(by_regs, by_smem), std::min(by_threads, by_tmem)));
        }
    }
    cache.push_back({{dev, (const void*)kern}, n});
    return n;
}

int um_heads(const FkvDecodeShape* sh, bool turbo);

struct KernelPick {
    KernelFn fn;
    int smem;
};

KernelPick pick_kernel(const FkvDecodeShape* sh, bool turbo, int nh) {
    if (turbo)
        return sh->D == 128 ? KernelPick{decode_fp8_kernel<128, kTurbo>, Ring<128, kTurbo>::BYTES + 1024}
                            : KernelPick{decode_fp8_kernel<64, kTurbo>, Ring<64, kTurbo>::BYTES + 1024};
    if (sh->D == 128) {
        if (nh == 4)
            return sh->v_group == 0 ? KernelPick{decode_fp8_kernel<128, 0, 4>, UmLayout<128, 0>::BYTES}
                                    : KernelPick{decode_fp8_kernel<128, 32, 4>, UmLayout<128, 32>::BYTES};
        if (nh == 8)
            return sh->v_group == 0 ? KernelPick{decode_fp8_kernel<128, 0, 8>, UmLayout<128, 0>::BYTES}
                                    : KernelPick{decode_fp8_kernel<128, 32, 8>, UmLayout<128, 32>::BYTES};
        return sh->v_group == 0 ? KernelPick{decode_fp8_kernel<128, 0>, Ring<128, 0>::BYTES + 1024}
                                : KernelPick{decode_fp8_kernel<128, 32>, Ring<128, 32>::BYTES + 1024};
    }
    return sh->v_group == 0 ? KernelPick{decode_fp8_kernel<64, 0>, Ring<64, 0>::BYTES + 1024}
                            : KernelPick{decode_fp8_kernel<64, 32>, Ring<64, 32>::BYTES + 1024};
}

// cluster-mode instantiations (mma.sync far path, or TurboQuant)
KernelPick pick_cl_kernel(const FkvDecodeShape* sh, bool turbo) {
    if (turbo)
        return sh->D == 128 ? KernelPick{decode_fp8_kernel<128, kTurbo, 0, true>, Ring<128, kTurbo>::BYTES + 1024}
                            : KernelPick{decode_fp8_kernel<64, kTurbo, 0, true>, Ring<64, kTurbo>::BYTES + 1024};
    if (sh->D == 128)
        return sh->v_group == 0 ? KernelPick{decode_fp8_kernel<128, 0, 0, true>, Ring<128, 0>::BYTES + 1024}
                                : KernelPick{decode_fp8_kernel<128, 32, 0, true>, Ring<128, 32>::BYTES + 1024};
    return sh->v_group == 0 ? KernelPick{decode_fp8_kernel<64, 0, 0, true>, Ring<64, 0>::BYTES + 1024}
                            : KernelPick{decode_fp8_kernel<64, 32, 0, true>, Ring<64, 32>::BYTES + 1024};
}

// Kernels that honour a caller wait limit and the stall test hook
// (FkvDecodeShape.wait_limit / test_flags): fp8 K with per-token INT4 V at
// D = 128, on both q.K paths.  Returns fn = nullptr for other shapes.
KernelPick pick_rt_kernel(const FkvDecodeShape* sh, bool turbo, int nh) {
    if (turbo || sh->D != 128 || sh->v_group != 0) return KernelPick{nullptr, 0};
    if (nh == 4) return KernelPick{decode_fp8_kernel<128, 0, 4, false, true>, UmLayout<128, 0>::BYTES};
    if (nh == 8) return KernelPick{decode_fp8_kernel<128, 0, 8, false, true>, UmLayout<128, 0>::BYTES};
    return KernelPick{decode_fp8_kernel<128, 0, 0, false, true>, Ring<128, 0>::BYTES + 1024};
}

int resident_for(const FkvDecodeShape* sh, bool turbo, int nh = -1) {
    if (nh < 0) nh = um_heads(sh, turbo);
    const KernelPick k = pick_kernel(sh, turbo, nh);
    return resident_ctas(k.fn, k.smem, nh > 0 ? (int)UmLayout<128, 0>::TMEM_COLS : 0);
}

// Tensor-map encoding (cuTensorMapEncodeTiled, resolved once through the
// runtime's driver entry point) with a small per-thread cache: a decode loop
// re-uses the same tier buffers call after call.
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q{};
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// 2-D map of a (rows, inner) row-major matrix with row pitch `pitch` bytes,
// read in (box_inner x box_rows) boxes with the 128-byte swizzle
bool encode_map(CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
                uint64_t pitch, uint32_t box_inner, uint32_t box_rows, CUtensorMap* out) {
    struct Entry {
        const void* base;
        uint64_t inner, rows, pitch;
        uint32_t bi, br;
        int dt;
        CUtensorMap map;
    };
    static thread_local std::vector<Entry> cache;
    for (const Entry& e : cache)
        if (e.base == base && e.inner == inner && e.rows == rows && e.pitch == pitch && e.bi == box_inner &&
            e.br == box_rows && e.dt == (int)dt) {
            *out = e.map;
            return true;
        }
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
    if (fn == nullptr || base == nullptr || rows == 0) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)pitch};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t es[2] = {1u, 1u};
    if (fn(out, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    if (cache.size() >= 64) cache.erase(cache.begin());
    cache.push_back(Entry{base, inner, rows, pitch, box_inner, box_rows, (int)dt, *out});
    return true;
}

// far K codes as a (B*Hk*F, D) byte matrix in boxes of 128 rows (the UMMA
// A-operand layout); false = unavailable (caller takes the mma.sync path)
bool far_k_tensor_map(const uint8_t* far_k, int64_t rows, int D, CUtensorMap* out) {
    return encode_map(CU_TENSOR_MAP_DATA_TYPE_UINT8, far_k, (uint64_t)D, (uint64_t)rows, (uint64_t)D,
                      (uint32_t)D, 128u, out);
}

// fp16 (rows, D) matrix (near tier, decode buffer) in boxes of 64 rows x 64
// halves (128 bytes)
bool fp16_tensor_map(const uint16_t* base, int64_t rows, int D, CUtensorMap* out) {
    return encode_map(CU_TENSOR_MAP_DATA_TYPE_UINT16, base, (uint64_t)D, (uint64_t)rows,
                      (uint64_t)D * 2, 64u, 64u, out);
}

struct Plan {
    int HG, splits, chunk;
    size_t rec_bytes, ticket_bytes;
    size_t qproj_bytes;   // turbo only: (B*Hq, 2D) f32 after the counters
    int near_w, far_w;
    int csize = 0, groups = 0;   // cluster mode (csize >= 2): CTAs per cluster, clusters per unit
};

// Cost model (measured on B200, per token): an fp16 near / decode token costs
// ~1.65x an fp8 / INT4 far token (weights 5 : 3) and ~0.8x a TurboQuant far
// token (4 : 5).  Fixed costs are in units of far tokens times far_w.
Plan make_plan(const FkvDecodeShape* sh, int resident, bool turbo = false) {
    Plan pl{};
    const int G = sh->Hq / sh->Hk;
    pl.HG = (G + kHeadsPerTile - 1) / kHeadsPerTile;
    pl.near_w = turbo ? 4 : 5;
    pl.far_w = turbo ? 5 : 3;
    const double fixed = (turbo ? 240.0 : 512.0) * pl.far_w, per_split = (turbo ? 3.0 : 8.0) * pl.far_w;
    // work of a (b, kv head) stream in cost units (the near tier counted at
    // its allocation; each CTA later splits its stream's actual rows)
    const int64_t T = pl.near_w * ((int64_t)sh->n_near_alloc + sh->n_dec) + (int64_t)pl.far_w * sh->n_far;
    const int64_t streams = (int64_t)sh->B * sh->Hk * pl.HG;
    int splits = sh->num_splits;
    if (splits <= 0) {
        // Pick the split count minimising the busiest SM's time.  The block
        // scheduler spreads the CTAs evenly over the SMs; each SM runs its
        // share in rounds of `resident` CTAs, a round of k co-resident CTAs
        // progressing at thr(k) CTA-speeds (measured on B200: thr(2) ~ 1.7;
        // thr(3) ~ 2.3 when the job is throughput-bound, but no better than 2
        // for small jobs, where the CTAs' start-up and merge latencies
        // dominate: c1 at S=4K..16K is fastest at 2 CTAs per SM).  Each CTA
        // also pays a fixed cost (launch, q fragments, pipeline fill, record
        // write), each split a small merge cost.
        const int nsm = num_sms();
        const int res = std::max(resident, 1);
        const bool small_job = (double)streams * (double)T / nsm < 60000.0;
        auto thr = [&](int k) { return k <= 1 ? 1.0 : (k == 2 || small_job) ? 1.7 : 2.3; };
        double best = 1e300;
        splits = 1;
        for (int sp = 1; sp <= 64; ++sp) {
            const int64_t chunk_tok = (T + sp - 1) / sp;
            if (sp > 1 && chunk_tok < 256 * pl.far_w) break;
            const int64_t per_sm = (streams * sp + nsm - 1) / nsm;
            const int64_t full = per_sm / res, rem = per_sm % res;
            const double cta = (double)chunk_tok + fixed;
            const double cost = (double)full * res * cta / thr(res) +
                                (rem ? (double)rem * cta / thr((int)rem) : 0.0) + per_split * sp;
            if (cost < best * 0.999) {
                best = cost;
                splits = sp;
            }
        }
    }
    splits = std::min(splits, kMaxSplits);
    int64_t chunk = (T + splits - 1) / splits;
    constexpr int64_t q = 64;   // chunk granularity (tokens)
    chunk = std::max<int64_t>(q, (chunk + q - 1) / q * q);
    pl.splits = (int)std::max<int64_t>(1, (T + chunk - 1) / chunk);
    pl.chunk = (int)chunk;
    const int D = sh->D;
    // split records, then (more than kDirectMerge splits) the group records
    // of the two-level merge; status word + one counter per stream, then the
    // group counters
    const int64_t ngrp = pl.splits > kDirectMerge ? (pl.splits + kMergeGroup - 1) / kMergeGroup : 0;
    pl.rec_bytes = pl.splits > 1 ? (size_t)streams * (pl.splits + ngrp) * (40 + 8 * D) * sizeof(float) : 0;
    pl.ticket_bytes = 16 + (size_t)streams * (1 + ngrp) * sizeof(int32_t);
    pl.qproj_bytes = (size_t)sh->B * sh->Hq * 2 * D * sizeof(float);
    return pl;
}

// Cluster mode plan.  Small jobs (fewer (stream, head group) units than half
// the resident CTA slots) give each unit one cluster of C CTAs, or m
// clusters of C (C <= 16), sized so that all clusters run in one wave and
// every CTA gets at least two ring stages; the CTAs of a cluster balance
// their stages dynamically and merge through distributed shared memory, the
// m cluster records of a unit (m > 1) through the workspace.  csize = 0:
// not eligible (large job, explicit split count, or no cluster fits).
bool cluster_mode_enabled() {
    // opt-in (FKV_CLUSTER=1): on B200 the flat split measured faster for
    // every benchmarked shape (the cluster placement leaves SMs idle)
    const char* e = std::getenv("FKV_CLUSTER");
    return e != nullptr && std::strcmp(e, "1") == 0;
}

// clusters of `c` CTAs of `k` that can run at once (0 = cannot launch)
int max_active_clusters(const KernelPick& k, int c, dim3 grid) {
    struct Entry {
        int dev;
        const void* fn;
        int c;
        int n;
    };
    static thread_local std::vector<Entry> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    for (const Entry& e : cache)
        if (e.dev == dev && e.fn == (const void*)k.fn && e.c == c) return e.n;
    int n = 0;
    if (cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem) == cudaSuccess &&
        cudaFuncSetAttribute(k.fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = k.smem;
        cudaLaunchAttribute a[1];
        a[0].id = cudaLaunchAttributeClusterDimension;
        a[0].val.clusterDim.x = (unsigned)c;
        a[0].val.clusterDim.y = 1;
        a[0].val.clusterDim.z = 1;
        cfg.attrs = a;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, k.fn, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();   // a failed query leaves no sticky error behind
    cache.push_back(Entry{dev, (const void*)k.fn, c, n});
    return n;
}

Plan make_cl_plan(const FkvDecodeShape* sh, bool turbo) {
    Plan pl = make_plan(sh, 2, turbo);
    pl.csize = pl.groups = 0;
    if (!cluster_mode_enabled() || sh->num_splits > 0) return pl;
    const KernelPick k = pick_cl_kernel(sh, turbo);
    const int res = resident_ctas(k.fn, k.smem);
    const int64_t units = (int64_t)sh->B * sh->Hk * pl.HG;
    const int64_t slots = (int64_t)num_sms() * res;
    if (units * 2 > slots) return pl;
    const int64_t stages = ((int64_t)sh->n_near_alloc + 63) / 64 + ((int64_t)sh->n_far + 127) / 128 +
                           ((int64_t)sh->n_dec + 63) / 64;
    const int64_t T = std::min<int64_t>(slots / units, std::max<int64_t>(1, stages / 2));
    if (T < 2) return pl;
    int C = (int)std::min<int64_t>(T, kMaxCluster);
    const int m = (int)std::max<int64_t>(1, std::min<int64_t>(T / C, kDirectMerge));
    // shrink the cluster until every cluster of the launch is co-resident
    for (; C >= 2; --C) {
        const dim3 grid((unsigned)(C * m), (unsigned)pl.HG, (unsigned)(sh->B * sh->Hk));
        if ((int64_t)max_active_clusters(k, C, grid) >= units * m) break;
    }
    if (C < 2) return pl;
    pl.csize = C;
    pl.groups = m;
    pl.splits = C * m;
    pl.rec_bytes = m > 1 ? (size_t)units * m * (40 + 8 * sh->D) * sizeof(float) : 0;
    return pl;
}

// q heads per CTA on the tensor-core far path (0 = mma.sync path).  Eligible:
// fp8 K with D = 128, a far tier, far rows inside the tensor map's int32
// range.  Chosen by default when a CTA's planned work is at least
// kUmMinChunk cost units: on B200 the tensor-core path's CTAs start (TMEM
// allocation, q pieces, first MMA) and drain about 3 us later while each far
// token costs a few percent less, and it takes the two-level split merge
// (c3, ~19K units per CTA: 633 vs 611 us; c4 2-GPU shards, ~30K per CTA:
// 168.4 vs 175.9 us per step; 4-GPU shards, ~23K: 106.3 vs 102.2; c4 on one
// GPU, ~61K: 312 vs 322 us).  FKV_QK_PATH=mma / tcgen05 forces either.
constexpr int64_t kUmMinChunk = 27000;

int um_heads(const FkvDecodeShape* sh, bool turbo) {
    if (turbo || sh->D != 128 || sh->n_far <= 0) return 0;
    if ((int64_t)sh->B * sh->Hk * sh->n_far >= ((int64_t)1 << 31) - 256) return 0;
    const int nh = (sh->Hq / sh->Hk) <= 4 ? 4 : 8;
    const char* e = std::getenv("FKV_QK_PATH");
    if (e != nullptr && std::strcmp(e, "mma") == 0) return 0;
    if (e != nullptr && std::strcmp(e, "tcgen05") == 0) return nh;
    const KernelPick k = pick_kernel(sh, false, nh);
    const Plan pl = make_plan(sh, resident_ctas(k.fn, k.smem, (int)UmLayout<128, 0>::TMEM_COLS));
    return pl.chunk >= kUmMinChunk ? nh : 0;
}

int validate(const FkvDecodeShape* sh) {
    FKV_REQUIRE(sh != nullptr, FKV_ERR_INVALID, "decode shape is NULL");
    FKV_REQUIRE(sh->B > 0 && sh->Hq > 0 && sh->Hk > 0, FKV_ERR_INVALID,
                "B=%d Hq=%d Hk=%d must be positive", sh->B, sh->Hq, sh->Hk);
    FKV_REQUIRE(sh->Hq % sh->Hk == 0, FKV_ERR_INVALID, "Hq=%d not a multiple of Hk=%d", sh->Hq,
                sh->Hk);
    FKV_REQUIRE(sh->D == 64 || sh->D == 128, FKV_ERR_UNSUPPORTED,
                "head dim %d unsupported (64, 128)", sh->D);
    FKV_REQUIRE(sh->n_near_alloc >= 0 && sh->n_far >= 0 && sh->n_dec >= 0 &&
                    sh->dec_stride >= sh->n_dec,
                FKV_ERR_INVALID, "bad tier sizes Np=%d F=%d n_dec=%d dec_stride=%d",
                sh->n_near_alloc, sh->n_far, sh->n_dec, sh->dec_stride);
    FKV_REQUIRE(sh->wait_limit >= 0 && (sh->test_flags & ~FKV_TEST_STALL) == 0, FKV_ERR_INVALID,
                "wait_limit=%d must be >= 0 and test_flags=%d a subset of FKV_TEST_STALL",
                sh->wait_limit, sh->test_flags);
    FKV_REQUIRE((int64_t)sh->B * sh->Hk <= 65535, FKV_ERR_UNSUPPORTED,
                "B*Hk=%lld exceeds the grid limit 65535", (long long)sh->B * sh->Hk);
    return FKV_OK;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// Opt every kernel instantiation into its dynamic shared memory once per
// device, then launch.
int launch_kernel(KernelFn kern, int smem, dim3 grid, const DecodeParams& p, cudaStream_t st,
                  const TMaps& maps, bool pdl = false, int cluster = 0) {
    static thread_local std::vector<std::pair<int, const void*>> done;
    int dev = 0;
    FKV_CUDA_CHECK(cudaGetDevice(&dev));
    const std::pair<int, const void*> key{dev, (const void*)kern};
    if (std::find(done.begin(), done.end(), key) == done.end()) {
        FKV_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        done.push_back(key);
    }
    if (cluster > 0) {
        // cluster mode (attributes set by max_active_clusters when planned)
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)cluster;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        FKV_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, p, maps));
    } else if (pdl) {
        // programmatic dependent launch: the decode grid may begin while the
        // previous kernel of the stream finishes -- after the q-projection
        // kernel its barrier set-up and first tier copies, after any other
        // kernel its set-up only (the kernel waits before any global read)
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        FKV_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, p, maps));
    } else {
        kern<<<grid, kThreads, smem, st>>>(p, maps);
    }
    FKV_LAUNCH_CHECK();
    return FKV_OK;
}

int launch(const FkvDecodeShape* sh, DecodeParams& p, void* workspace, size_t ws_bytes,
           cudaStream_t st, bool turbo = false) {
    int nh = um_heads(sh, turbo);
    TMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    if (nh > 0 && !far_k_tensor_map(p.far_k, (int64_t)sh->B * sh->Hk * sh->n_far, sh->D, &maps.far_k))
        nh = 0;
    {
        const int64_t bh = (int64_t)sh->B * sh->Hk;
        FKV_REQUIRE(bh * std::max(sh->n_near_alloc, sh->dec_stride) < ((int64_t)1 << 31), FKV_ERR_UNSUPPORTED,
                    "near / decode rows exceed the tensor-map coordinate range");
        if (sh->n_near_alloc > 0)
            FKV_REQUIRE(fp16_tensor_map(p.near_k, bh * sh->n_near_alloc, sh->D, &maps.near_k) &&
                            fp16_tensor_map(p.near_v, bh * sh->n_near_alloc, sh->D, &maps.near_v),
                        FKV_ERR_CUDA, "cuTensorMapEncodeTiled failed for the near tier");
        if (sh->n_dec > 0)
            FKV_REQUIRE(fp16_tensor_map(p.dec_k, bh * sh->dec_stride, sh->D, &maps.dec_k) &&
                            fp16_tensor_map(p.dec_v, bh * sh->dec_stride, sh->D, &maps.dec_v),
                        FKV_ERR_CUDA, "cuTensorMapEncodeTiled failed for the decode buffer");
    }
    KernelPick kp = pick_kernel(sh, turbo, nh);
    Plan pl = make_plan(sh, resident_ctas(kp.fn, kp.smem, nh > 0 ? (int)UmLayout<128, 0>::TMEM_COLS : 0), turbo);
    if (nh == 0) {
        const Plan cp = make_cl_plan(sh, turbo);
        if (cp.csize >= 2) {
            pl = cp;
            kp = pick_cl_kernel(sh, turbo);
        }
    }
    const bool cl = pl.csize >= 2;
    if (sh->wait_limit != 0 || sh->test_flags != 0) {
        FKV_REQUIRE(!cl, FKV_ERR_UNSUPPORTED, "wait_limit / test_flags are not honoured in cluster mode");
        const KernelPick rk = pick_rt_kernel(sh, turbo, nh);
        FKV_REQUIRE(rk.fn != nullptr, FKV_ERR_UNSUPPORTED,
                    "wait_limit / test_flags need D = 128 with per-token INT4 V (fp8 far tier)");
        kp = rk;   // same layout, plan and residency as the kernel it replaces
    }
    const size_t qoff = (pl.ticket_bytes + 255) & ~(size_t)255;
    const size_t front = turbo && !cl ? qoff + pl.qproj_bytes : pl.ticket_bytes;
    const size_t need = pl.rec_bytes + front + 256;
    FKV_REQUIRE(workspace != nullptr && ws_bytes >= need, FKV_ERR_INVALID,
                "workspace too small: %zu < %zu bytes", ws_bytes, need);
    FKV_REQUIRE(aligned16(workspace), FKV_ERR_INVALID, "workspace must be 16-byte aligned");
    p.B = sh->B; p.Hq = sh->Hq; p.Hk = sh->Hk; p.G = sh->Hq / sh->Hk; p.HG = pl.HG;
    p.Np = sh->n_near_alloc; p.F = sh->n_far; p.n_dec = sh->n_dec; p.dec_stride = sh->dec_stride;
    p.splits = pl.splits; p.near_w = pl.near_w; p.far_w = pl.far_w; p.margin = sh->spike_margin;
    p.csize = pl.csize; p.groups = pl.groups;
    p.qscale = (float)(1.0 / sqrt((double)sh->D));   // same f32 constant as the host oracle
    p.wait_limit = sh->wait_limit > 0 ? (uint32_t)sh->wait_limit : kWaitLimit;
    p.test_stall = (sh->test_flags & FKV_TEST_STALL) ? 1 : 0;
    // split counters at the front, split records at the back: a workspace
    // shared by calls of different shapes keeps every counter at zero as long
    // as it holds the largest records region plus the largest counter region.
    p.status = reinterpret_cast<int32_t*>(workspace);
    p.tickets = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(workspace) + 16);
    const size_t rec_off = (ws_bytes - pl.rec_bytes) & ~(size_t)255;
    FKV_REQUIRE(rec_off >= front, FKV_ERR_INVALID,
                "workspace too small for counters + records (%zu bytes)", ws_bytes);
    p.ws = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + rec_off);
    dim3 grid(pl.splits, pl.HG, sh->B * sh->Hk);
    if (cl) return launch_kernel(kp.fn, kp.smem, grid, p, st, maps, false, pl.csize);
    if (turbo) {
        float* qproj = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + qoff);
        p.qproj = qproj;
        const int BH = sh->B * sh->Hq;
        FKV_REQUIRE((BH + kQpHeads - 1) / kQpHeads <= 65535, FKV_ERR_UNSUPPORTED,
                    "B*Hq=%d exceeds the q-projection grid limit", BH);
        const dim3 qg(2 * sh->D / kQpRows, (BH + kQpHeads - 1) / kQpHeads);
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = qg;
        cfg.blockDim = dim3(kQpThreads);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (sh->D == 128)
            FKV_CUDA_CHECK(cudaLaunchKernelEx(&cfg, turbo_qproj_kernel<128>, p.q, p.turbo_pi, p.turbo_s,
                                              qproj, BH));
        else
            FKV_CUDA_CHECK(cudaLaunchKernelEx(&cfg, turbo_qproj_kernel<64>, p.q, p.turbo_pi, p.turbo_s,
                                              qproj, BH));
        FKV_LAUNCH_CHECK();
    }
    // Early start only for grids of at most one CTA per SM: their CTAs land
    // on whichever SMs the previous kernel frees first without crowding.
    // Larger grids launched early were placed unevenly over the SMs (the
    // SMs that finished first took several CTAs) and ran slower: c1 at 16K,
    // 288 CTAs, 32.2 -> 40.2 us per layer; c0 gained 8.0 -> 7.0 us.
    const bool early = turbo || (int64_t)grid.x * grid.y * grid.z <= num_sms();
    return launch_kernel(kp.fn, kp.smem, grid, p, st, maps, early);
}

int fill_common(const FkvDecodeShape* sh, DecodeParams& p, const uint16_t* near_k,
                const uint16_t* near_v, const int32_t* near_valid, const uint8_t* far_k,
                const uint8_t* far_v, const uint16_t* v_scale, const uint16_t* v_zero,
                const uint16_t* q, const uint16_t* dec_k, const uint16_t* dec_v) {
    int rc = validate(sh);
    if (rc) return rc;
    FKV_REQUIRE(sh->v_group == 0 || sh->v_group == 32, FKV_ERR_UNSUPPORTED,
                "v_group=%d unsupported (0, 32)", sh->v_group);
    FKV_REQUIRE(q && near_valid, FKV_ERR_INVALID, "q / near_valid is NULL");
    FKV_REQUIRE(sh->n_near_alloc == 0 || (near_k && near_v), FKV_ERR_INVALID, "near is NULL");
    FKV_REQUIRE(sh->n_far == 0 || (far_k && far_v && v_scale && v_zero), FKV_ERR_INVALID,
                "far tier pointer is NULL");
    FKV_REQUIRE(sh->n_dec == 0 || (dec_k && dec_v), FKV_ERR_INVALID, "decode buffer is NULL");
    FKV_REQUIRE(aligned16(q) && aligned16(near_k) && aligned16(near_v) && aligned16(far_k) &&
                    aligned16(dec_k) && aligned16(dec_v) && aligned16(far_v) &&
                    ((uintptr_t)v_scale & 1u) == 0 && ((uintptr_t)v_zero & 1u) == 0,
                FKV_ERR_INVALID, "tier / query pointers misaligned");
    p = DecodeParams{};
    p.near_k = near_k; p.near_v = near_v; p.near_valid = near_valid;
    p.far_k = far_k; p.far_v = far_v; p.v_scale = v_scale; p.v_zero = v_zero;
    p.q = q; p.dec_k = dec_k; p.dec_v = dec_v;
    return FKV_OK;
}

}  // namespace

extern "C" {

size_t fkv_decode_workspace_bytes(const FkvDecodeShape* s) {
    if (validate(s) != FKV_OK) return 0;
    // enough for either far-tier kind (their resident counts, hence split
    // counts, may differ)
    // (and for either q.K path of the fp8 tier)
    const Plan a = make_plan(s, resident_for(s, false)), b = make_plan(s, resident_for(s, true), true);
    const Plan c = make_plan(s, resident_for(s, false, 0));
    const Plan d = make_cl_plan(s, false), e = make_cl_plan(s, true);
    size_t rec = 0, tick = 0, qp = 0;
    for (const Plan* pl : {&a, &b, &c, &d, &e}) {
        rec = std::max(rec, pl->rec_bytes);
        tick = std::max(tick, pl->ticket_bytes);
        qp = std::max(qp, pl->qproj_bytes);
    }
    return rec + tick + 256 + ((qp + 255) & ~(size_t)255) + 256;
}

int fkv_decode_status(const void* workspace, int32_t* status, int32_t clear, void* stream) {
    fkv::clear_error();
    FKV_REQUIRE(workspace != nullptr && status != nullptr, FKV_ERR_INVALID,
                "fkv_decode_status: NULL argument");
    FKV_REQUIRE(aligned16(workspace), FKV_ERR_INVALID, "workspace must be 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    int32_t word = 0;
    FKV_CUDA_CHECK(cudaMemcpyAsync(&word, workspace, sizeof(word), cudaMemcpyDeviceToHost, st));
    FKV_CUDA_CHECK(cudaStreamSynchronize(st));
    if (clear && word != 0)
        FKV_CUDA_CHECK(cudaMemsetAsync(const_cast<void*>(workspace), 0, sizeof(word), st));
    *status = word;
    return FKV_OK;
}

int fkv_decode_plan(const FkvDecodeShape* sh, const uint8_t* far_k, int32_t turbo, int32_t* out) {
    fkv::clear_error();
    const int rc = validate(sh);
    if (rc) return rc;
    FKV_REQUIRE(out != nullptr, FKV_ERR_INVALID, "fkv_decode_plan: out is NULL");
    int nh = turbo ? 0 : um_heads(sh, false);
    if (nh > 0) {
        CUtensorMap m;
        if (far_k == nullptr || !aligned16(far_k) ||
            !far_k_tensor_map(far_k, (int64_t)sh->B * sh->Hk * sh->n_far, sh->D, &m))
            nh = 0;
    }
    const KernelPick kp = pick_kernel(sh, turbo != 0, nh);
    Plan pl = make_plan(sh, resident_ctas(kp.fn, kp.smem, nh > 0 ? (int)UmLayout<128, 0>::TMEM_COLS : 0),
                        turbo != 0);
    if (nh == 0) {
        const Plan cp = make_cl_plan(sh, turbo != 0);
        if (cp.csize >= 2) pl = cp;
    }
    out[0] = nh;
    out[1] = pl.splits;
    out[2] = pl.csize;
    out[3] = pl.groups;
    return FKV_OK;
}

int fkv_decode_qk_path(const FkvDecodeShape* sh, const uint8_t* far_k) {
    const int rc = validate(sh);
    if (rc) return rc;
    const int nh = um_heads(sh, false);
    if (nh == 0) return 0;
    FKV_REQUIRE(far_k != nullptr && aligned16(far_k), FKV_ERR_INVALID, "far_k NULL or misaligned");
    CUtensorMap m;
    return far_k_tensor_map(far_k, (int64_t)sh->B * sh->Hk * sh->n_far, sh->D, &m) ? nh : 0;
}

int fkv_decode_fp8(const FkvDecodeShape* sh, const uint16_t* near_k, const uint16_t* near_v,
                   const int32_t* near_valid, const uint8_t* far_k, const uint8_t* far_v,
                   const uint16_t* v_scale, const uint16_t* v_zero, const uint16_t* q,
                   const uint16_t* dec_k, const uint16_t* dec_v, uint16_t* out,
                   int32_t* flags, int32_t* tokens, void* workspace, size_t workspace_bytes,
                   void* stream) {
    fkv::clear_error();
    DecodeParams p;
    int rc = fill_common(sh, p, near_k, near_v, near_valid, far_k, far_v, v_scale, v_zero, q,
                         dec_k, dec_v);
    if (rc) return rc;
    FKV_REQUIRE(out && flags && tokens, FKV_ERR_INVALID, "outputs are NULL");
    FKV_REQUIRE(aligned16(out), FKV_ERR_INVALID, "out must be 16-byte aligned");
    p.out = out; p.flags = flags; p.tokens = tokens;
    return launch(sh, p, workspace, workspace_bytes, (cudaStream_t)stream);
}

int fkv_decode_turbo(const FkvDecodeShape* sh, const uint16_t* near_k, const uint16_t* near_v,
                     const int32_t* near_valid, const uint8_t* k_idx, const uint8_t* k_signs,
                     const uint16_t* k_norm, const uint16_t* k_gamma, const uint8_t* v_packed,
                     const uint16_t* v_scale, const float* Pi, const float* Smat,
                     const float* centroids, const uint16_t* q, const uint16_t* dec_k,
                     const uint16_t* dec_v, uint16_t* out, int32_t* flags, int32_t* tokens,
                     void* workspace, size_t workspace_bytes, void* stream) {
    fkv::clear_error();
    int rc = validate(sh);
    if (rc) return rc;
    FKV_REQUIRE(q && near_valid && Pi && Smat && centroids && out && flags && tokens,
                FKV_ERR_INVALID, "fkv_decode_turbo: NULL argument");
    FKV_REQUIRE(sh->n_near_alloc == 0 || (near_k && near_v), FKV_ERR_INVALID, "near is NULL");
    FKV_REQUIRE(sh->n_far == 0 || (k_idx && k_signs && k_norm && k_gamma && v_packed && v_scale),
                FKV_ERR_INVALID, "turbo far tier pointer is NULL");
    FKV_REQUIRE(sh->n_dec == 0 || (dec_k && dec_v), FKV_ERR_INVALID, "decode buffer is NULL");
    FKV_REQUIRE(aligned16(q) && aligned16(near_k) && aligned16(near_v) && aligned16(k_idx) &&
                    aligned16(v_packed) && aligned16(dec_k) && aligned16(dec_v) &&
                    ((uintptr_t)k_signs & 3u) == 0,
                FKV_ERR_INVALID, "turbo tier / query pointers misaligned");
    DecodeParams p{};
    p.near_k = near_k; p.near_v = near_v; p.near_valid = near_valid;
    p.far_k = k_idx; p.far_v = v_packed; p.v_scale = v_scale;
    p.k_signs = k_signs; p.k_norm = k_norm; p.k_gamma = k_gamma; p.centroids = centroids;
    p.turbo_pi = Pi; p.turbo_s = Smat; p.qjl_coef = sh->qjl_coef;
    p.q = q; p.dec_k = dec_k; p.dec_v = dec_v;
    FKV_REQUIRE(aligned16(out), FKV_ERR_INVALID, "out must be 16-byte aligned");
    p.out = out; p.flags = flags; p.tokens = tokens;
    return launch(sh, p, workspace, workspace_bytes, (cudaStream_t)stream, true);
}

int fkv_decode_fp8_partial(const FkvDecodeShape* sh, const uint16_t* near_k,
                           const uint16_t* near_v, const int32_t* near_valid,
                           const uint8_t* far_k, const uint8_t* far_v, const uint16_t* v_scale,
                           const uint16_t* v_zero, const uint16_t* q, const uint16_t* dec_k,
                           const uint16_t* dec_v, int32_t far_index_offset, float* part,
                           int32_t* part_arg, void* workspace, size_t workspace_bytes,
                           void* stream) {
    fkv::clear_error();
    DecodeParams p;
    int rc = fill_common(sh, p, near_k, near_v, near_valid, far_k, far_v, v_scale, v_zero, q,
                         dec_k, dec_v);
    if (rc) return rc;
    FKV_REQUIRE(part && part_arg, FKV_ERR_INVALID, "partial outputs are NULL");
    FKV_REQUIRE(aligned16(part), FKV_ERR_INVALID, "part must be 16-byte aligned");
    p.part = part; p.part_arg = part_arg; p.far_offset = far_index_offset;
    return launch(sh, p, workspace, workspace_bytes, (cudaStream_t)stream);
}

int fkv_combine_partials_strided(int32_t P, int32_t N, int32_t D, const float* parts,
                                 int64_t part_rank_stride, const int32_t* part_args,
                                 int64_t arg_rank_stride, float spike_margin, uint16_t* out,
                                 int32_t* flags, int32_t* tokens, void* stream) {
    fkv::clear_error();
    FKV_REQUIRE(P > 0 && N > 0, FKV_ERR_INVALID, "P=%d N=%d must be positive", P, N);
    FKV_REQUIRE(D == 64 || D == 128, FKV_ERR_UNSUPPORTED, "head dim %d unsupported", D);
    FKV_REQUIRE(parts && part_args && out && flags && tokens, FKV_ERR_INVALID, "NULL argument");
    FKV_REQUIRE(part_rank_stride >= (int64_t)N * (D + 4) && arg_rank_stride >= N, FKV_ERR_INVALID,
                "rank strides %lld / %lld smaller than one shard's records",
                (long long)part_rank_stride, (long long)arg_rank_stride);
    if (D == 128)
        combine_kernel<128><<<N, 128, 0, (cudaStream_t)stream>>>(
            P, N, parts, part_rank_stride, part_args, arg_rank_stride, spike_margin, out, flags, tokens);
    else
        combine_kernel<64><<<N, 64, 0, (cudaStream_t)stream>>>(
            P, N, parts, part_rank_stride, part_args, arg_rank_stride, spike_margin, out, flags, tokens);
    FKV_LAUNCH_CHECK();
    return FKV_OK;
}

int fkv_combine_partials(int32_t P, int32_t N, int32_t D, const float* parts,
                         const int32_t* part_args, float spike_margin, uint16_t* out,
                         int32_t* flags, int32_t* tokens, void* stream) {
    return fkv_combine_partials_strided(P, N, D, parts, (int64_t)N * (D + 4), part_args, N,
                                        spike_margin, out, flags, tokens, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of fkv_decode_fp8
// ---------------------------------------------------------------------------
// Some callers cannot allocate device memory at the point where they decode:
// code running under an allocator that is locked or owned by someone else
// (an inference server's pre-planned memory pool, a plugin host that hands
// out only the tensors it manages), or a runtime that forbids cudaMalloc on
// the decode path.  For them the split-K scratch lives in this fixed
// file-scope device array instead of a caller workspace.
namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;   // 16 MiB per GPU, held until exit
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// The array belongs to the CUDA context that loaded this module, so its
// address is cached per context (the current context, resolved through the
// runtime's driver entry point), not per device ordinal: a plugin host that
// drives its own contexts, or a process that resets a device, gets a fresh
// lookup instead of a stale address.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
struct ScratchEntry {
    CUcontext ctx;
    void* ptr;
};
std::vector<ScratchEntry> g_scratch;
std::mutex g_scratch_mu;

CtxGetCurrentFn ctx_get_current_fn() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q{};
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(f);
    });
    return fn;
}

// Device address of the scratch array in the current context.  The array's
// host-side name is only a stand-in: the address must come from
// cudaGetSymbolAddress, queried with the device (context) current.
int noalloc_scratch(void** out) {
    int dev = 0;
    FKV_CUDA_CHECK(cudaGetDevice(&dev));
    CtxGetCurrentFn get = ctx_get_current_fn();
    FKV_REQUIRE(get != nullptr, FKV_ERR_CUDA, "cuCtxGetCurrent unavailable");
    CUcontext ctx = nullptr;
    FKV_REQUIRE(get(&ctx) == CUDA_SUCCESS, FKV_ERR_CUDA, "cuCtxGetCurrent failed");
    if (ctx == nullptr) {
        // no context yet: a runtime call that needs one makes the device's
        // primary context current
        void* probe = nullptr;
        FKV_CUDA_CHECK(cudaGetSymbolAddress(&probe, g_noalloc_scratch));
        FKV_REQUIRE(get(&ctx) == CUDA_SUCCESS && ctx != nullptr, FKV_ERR_CUDA,
                    "no current CUDA context on device %d", dev);
    }
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    for (const ScratchEntry& e : g_scratch)
        if (e.ctx == ctx) {
            *out = e.ptr;
            return FKV_OK;
        }
    void* p = nullptr;
    FKV_CUDA_CHECK(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_scratch.push_back(ScratchEntry{ctx, p});
    *out = p;
    return FKV_OK;
}

}  // namespace

extern "C" int fkv_decode_fp8_noalloc(const FkvDecodeShape* sh, const uint16_t* near_k,
                                      const uint16_t* near_v, const int32_t* near_valid,
                                      const uint8_t* far_k, const uint8_t* far_v,
                                      const uint16_t* v_scale, const uint16_t* v_zero,
                                      const uint16_t* q, const uint16_t* dec_k,
                                      const uint16_t* dec_v, uint16_t* out, int32_t* flags,
                                      int32_t* tokens, void* stream) {
    fkv::clear_error();
    int rc = validate(sh);
    if (rc) return rc;
    // the launch may take either q.K path (the tensor-core one falls back to
    // mma.sync when far_k has no tensor map): accept only shapes whose
    // scratch fits for both, so the check below is the exact limit
    const Plan pa = make_plan(sh, resident_for(sh, false)), pb = make_plan(sh, resident_for(sh, false, 0));
    const Plan pc = make_cl_plan(sh, false);
    const Plan& pab = pa.rec_bytes + pa.ticket_bytes >= pb.rec_bytes + pb.ticket_bytes ? pa : pb;
    const Plan& pl = pab.rec_bytes + pab.ticket_bytes >= pc.rec_bytes + pc.ticket_bytes ? pab : pc;
    const size_t need = pl.rec_bytes + pl.ticket_bytes + 256;
    FKV_REQUIRE(need <= kNoAllocScratchBytes, FKV_ERR_INVALID,
                "fkv_decode_fp8_noalloc: shape needs %zu scratch bytes, above the fixed "
                "%zu-byte limit; use fkv_decode_fp8 with a caller workspace",
                need, kNoAllocScratchBytes);
    void* scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    // the array keeps the previous call's contents: zero the status word and
    // split counters (the front of the scratch) before this call uses them
    FKV_CUDA_CHECK(cudaMemsetAsync(scratch, 0, pl.ticket_bytes, (cudaStream_t)stream));
    return fkv_decode_fp8(sh, near_k, near_v, near_valid, far_k, far_v, v_scale, v_zero, q,
                          dec_k, dec_v, out, flags, tokens, scratch, kNoAllocScratchBytes,
                          stream);
}

extern "C" int fkv_decode_noalloc_status(int32_t* status, void* stream) {
    fkv::clear_error();
    FKV_REQUIRE(status != nullptr, FKV_ERR_INVALID, "fkv_decode_noalloc_status: status is NULL");
    void* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    return fkv_decode_status(scratch, status, 0, stream);
}
