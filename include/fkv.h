/*
 * fkv.h -- C ABI of libfkv.so, the B200 (sm_100a) FoveatedKV decode hot path.
 *
 * Plain pointers and sizes only.  Device pointers are raw CUDA device
 * addresses; fp16 tensors are passed as uint16_t* (IEEE binary16 bits).
 * ``stream`` is a cudaStream_t passed as void* (NULL = legacy default stream).
 * Every entry returns 0 on success or a negative FKV_ERR_* code; the message
 * of the last failure on the calling thread is returned by fkv_last_error().
 * No decode or compress entry point allocates device memory: scratch space
 * ("workspace") is passed in by the caller, sized by the matching
 * *_workspace_bytes() call.  The promotion pipeline (fkv_promo_*) owns its
 * pinned host staging and one device staging buffer, allocated and grown by
 * its worker thread.
 *
 * Each declaration cites the reference interface it replaces
 * (samfurr/foveated_kv 0.2.0, path within that project).
 */
#ifndef FKV_H_
#define FKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FKV_OK 0
#define FKV_ERR_INVALID (-1)     /* bad argument / shape */
#define FKV_ERR_UNSUPPORTED (-2) /* valid but not supported (e.g. head dim) */
#define FKV_ERR_CUDA (-3)        /* CUDA runtime error */
#define FKV_ERR_TIMEOUT (-4)     /* bounded wait expired */
#define FKV_ERR_IO (-5)          /* file / mmap failure */

/* Version of this ABI (bumped on any signature change). */
int fkv_abi_version(void);

/* Message of the last failure on this thread ("" if none). */
const char* fkv_last_error(void);

/* ------------------------------------------------------------------------ */
/* Tier layout                                                              */
/* ------------------------------------------------------------------------ */

/* Mirrors the dict returned by MLXTierConfig.tier_boundaries. */
typedef struct FkvTierLayout {
    int32_t S;               /* prefill length */
    int32_t n_sinks;
    int32_t window;
    int32_t near_from_mid;
    int32_t far_count;       /* F */
    int32_t r_actual;        /* R: valid near rows after compression */
    int32_t n_near_padded;   /* Np = R + headroom */
    int32_t mid_start;
    int32_t mid_end;
    int32_t near_mid_start;
} FkvTierLayout;

/* Replaces MLXTierConfig.tier_boundaries (src/foveated_kv/mlx_foveated.py:128-169)
 * and its C++ copy (csrc/foveated_compress.cpp:107-126).  Host only. */
int fkv_tier_boundaries(int32_t S, double near_pct, int32_t n_sinks, int32_t window_size,
                        double promo_headroom_pct, int32_t promo_headroom_min,
                        FkvTierLayout* out);

/* ------------------------------------------------------------------------ */
/* Tier selection + compression (prefill -> tiers)                          */
/* ------------------------------------------------------------------------ */

/* Recency selection: fills near_idx (B,Hk,Np) (-1 in headroom), far_idx
 * (B,Hk,F) and near_valid (B,Hk) = R.  Replaces the index construction of
 * _assign_and_build_layer (src/foveated_kv/mlx_foveated.py:823-843,907-917). */
int fkv_select_recency(const FkvTierLayout* L, int32_t B, int32_t Hk, int32_t* near_idx,
                       int32_t* far_idx, int32_t* near_valid, void* stream);

/* Importance selection (no reference implementation; the reference selects by
 * recency only).  Per KV head: sinks and window stay near; the near_from_mid
 * middle tokens with the largest sum over the G query heads of
 * softmax(q_obs . k / sqrt(D)) (fp64) are near, ties to the lower position.
 * k: (B,Hk,*,D) fp16 with kv_stride_bh elements between (b,h) rows of S tokens;
 * q_obs: (B,Hq,D) fp16. */
size_t fkv_select_importance_workspace_bytes(const FkvTierLayout* L, int32_t B, int32_t Hk,
                                             int32_t Hq);
int fkv_select_importance(const FkvTierLayout* L, int32_t B, int32_t Hk, int32_t Hq, int32_t D,
                          const uint16_t* k, int64_t kv_stride_bh, const uint16_t* q_obs,
                          int32_t* near_idx, int32_t* far_idx, int32_t* near_valid,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Gather + fp8/INT4 encode + archive scatter in one pass.  Replaces
 * CompressHandle::compress_layer (csrc/foveated_compress.cpp:95-201) and the
 * Metal kernels compress_foveal / compress_fp8 / compress_int4
 * (csrc/kernels/foveated_compress.metal:39-205), with the Python CPU path's
 * code semantics (mlx_foveated.py:528-600).
 *   k, v      (B,Hk,*,D) fp16, kv_stride_bh elements between (b,h) rows
 *   near_idx  (B,Hk,Np), far_idx (B,Hk,F) from fkv_select_*
 *   near_k/v  (B,Hk,Np,D) fp16 out (headroom rows zeroed)
 *   far_k     (B,Hk,F,D) u8 E4M3;  far_v (B,Hk,F,D/2) u8 nibbles
 *   v_scale/v_zero  (B,Hk,F) fp16 if v_group==0 (per token, the reference),
 *                   (B,Hk,F,D/v_group) if v_group==32
 *   arc_k/arc_v (B,Hk,F,D) fp16 exact copies of far rows, may be NULL. */
int fkv_compress_fp8(const FkvTierLayout* L, int32_t B, int32_t Hk, int32_t D,
                     const uint16_t* k, const uint16_t* v, int64_t kv_stride_bh,
                     const int32_t* near_idx, const int32_t* far_idx, int32_t v_group,
                     uint16_t* near_k, uint16_t* near_v, uint8_t* far_k, uint8_t* far_v,
                     uint16_t* v_scale, uint16_t* v_zero, uint16_t* arc_k, uint16_t* arc_v,
                     void* stream);

/* TurboQuant far tier.  Replaces turbo_compress_keys / turbo_compress_values
 * (src/foveated_kv/turbo_quantize.py:25-178) on the _assign_and_build_layer
 * path (mlx_foveated.py:869-894); fp64 accumulation.
 *   Pi, Smat (D,D) f32 row-major; centroids[4], boundaries[3] f32
 *   k_idx (B,Hk,F,D/4) u8; k_signs (B,Hk,F,D/8) u8; k_norm, k_gamma (B,Hk,F) fp16
 *   v_packed (B,Hk,F,D/4) u8; v_scale (B,Hk,F,D/32) fp16 */
int fkv_compress_turbo(const FkvTierLayout* L, int32_t B, int32_t Hk, int32_t D,
                       const uint16_t* k, const uint16_t* v, int64_t kv_stride_bh,
                       const int32_t* near_idx, const int32_t* far_idx,
                       const float* Pi, const float* Smat, const float* centroids,
                       const float* boundaries, uint16_t* near_k, uint16_t* near_v,
                       uint8_t* k_idx, uint8_t* k_signs, uint16_t* k_norm, uint16_t* k_gamma,
                       uint8_t* v_packed, uint16_t* v_scale, uint16_t* arc_k, uint16_t* arc_v,
                       void* stream);

/* ------------------------------------------------------------------------ */
/* Fused two-tier decode attention with spike emission                      */
/* ------------------------------------------------------------------------ */

typedef struct FkvDecodeShape {
    int32_t B, Hq, Hk, D;
    int32_t n_near_alloc;  /* Np: rows per (b,h) of near_k/near_v */
    int32_t n_far;         /* F */
    int32_t n_dec;         /* valid decode-buffer tokens */
    int32_t dec_stride;    /* decode-buffer capacity (rows per (b,h)), >= n_dec */
    int32_t v_group;       /* fp8 mode: 0 = per-token INT4 V scales, 32 = grouped */
    int32_t num_splits;    /* split-K chunks per (b,h); 0 = automatic */
    float spike_margin;    /* flag = max_far > min_near + spike_margin */
    float qjl_coef;        /* turbo only: QJL term = qjl_coef/D * gamma * <sign, q S^T> */
    /* wait_limit / test_flags: honoured for fp8 K with per-token INT4 V at
       D = 128 outside the cluster mode; other shapes return FKV_ERR_UNSUPPORTED
       when either is set. */
    int32_t wait_limit;    /* iteration limit of the kernel's progress waits; 0 = default
                              (2^26).  On expiry the kernel records FKV_ERR_TIMEOUT in the
                              workspace status word (fkv_decode_status), lets its copies
                              in flight land and exits. */
    int32_t test_flags;    /* 0 in normal use.  FKV_TEST_STALL: the consumers first wait on
                              a barrier that nothing completes, so a test can drive the
                              timeout path (with a small wait_limit) without any fault. */
} FkvDecodeShape;

#define FKV_TEST_STALL 1

/* Scratch bytes for fkv_decode_fp8 / fkv_decode_turbo / fkv_decode_fp8_partial:
 * split counters (4 bytes per (b, kv head, group of 8 q heads)) at the front
 * of the workspace, split records at its back.  The workspace must be
 * zero-filled once before first use; the kernels return the counters to zero.
 * One workspace may serve calls of different shapes if it is at least
 * (largest records region + largest counter region + 256) bytes, i.e. the sum
 * of the two largest values this function returned for them.  Calls that
 * share a workspace must not overlap on the GPU. */
size_t fkv_decode_workspace_bytes(const FkvDecodeShape* s);

/* One fused launch per layer: near fp16 (rows [0, near_valid[b,h])) + far
 * fp8 E4M3 K / INT4 V + decode buffer, split-K with in-launch combine, and
 * spike flags / tokens.  Replaces FoveatedHandle::operator()
 * (csrc/foveated_attn.cpp:164-240) and kernel foveated_2tier
 * (csrc/kernels/foveated_attn.metal:181-432).
 *   near_k/near_v (B,Hk,Np,D) fp16; near_valid (B,Hk) int32, read by every
 *   CTA of the launch: it must not change while the launch runs (when a
 *   promotion worker may bump it concurrently, pass a copy taken in stream
 *   order just before the call, as FoveatedLayer does once registered)
 *   far_k (B,Hk,F,D) u8; far_v (B,Hk,F,D/2) u8; v_scale/v_zero as compress
 *   q (B,Hq,D) fp16; dec_k/dec_v (B,Hk,dec_stride,D) fp16 (NULL if n_dec==0)
 *   out (B,Hq,D) fp16, 16-byte aligned; flags (B,Hq) int32; tokens (B,Hq)
 *   int32 far-local or -1 */
int fkv_decode_fp8(const FkvDecodeShape* s, const uint16_t* near_k, const uint16_t* near_v,
                   const int32_t* near_valid, const uint8_t* far_k, const uint8_t* far_v,
                   const uint16_t* v_scale, const uint16_t* v_zero, const uint16_t* q,
                   const uint16_t* dec_k, const uint16_t* dec_v, uint16_t* out,
                   int32_t* flags, int32_t* tokens, void* workspace, size_t workspace_bytes,
                   void* stream);

/* Kernel status word of the decode calls that used `workspace` (no
 * counterpart in the reference, whose Metal kernels have no bounded waits):
 * waits for `stream`, then *status = 0 or FKV_ERR_TIMEOUT (a bounded wait
 * expired in some launch since the word was last cleared; that launch's
 * outputs are not valid).  The word is sticky across launches; clear != 0
 * resets it to 0 (stream-ordered).  Returns FKV_OK or an error of the read. */
int fkv_decode_status(const void* workspace, int32_t* status, int32_t clear, void* stream);

/* Which q.K path fkv_decode_fp8 / _partial / _noalloc take for this shape
 * and far_k pointer (no counterpart in the reference, whose Metal kernel has
 * one path): 4 or 8 = q heads per CTA on the 5th-generation tensor cores
 * (tcgen05.mma on the E4M3 codes, scores in tensor memory), 0 = mma.sync
 * after converting the codes, negative = invalid shape.  The tensor-core
 * path needs D = 128 and a far tier; by default it is taken when the planned
 * work per CTA is large (its CTAs start and drain a little later but process
 * far tokens a little faster).  The environment variable FKV_QK_PATH=mma or
 * FKV_QK_PATH=tcgen05 forces either path where the shape allows it. */
int fkv_decode_qk_path(const FkvDecodeShape* s, const uint8_t* far_k);

/* How a decode call of this shape is launched (no counterpart in the
 * reference): out[0] = q heads per CTA on the tensor-core q.K path (0 =
 * mma.sync), out[1] = CTAs per (b, kv head, group of 8 q heads), out[2] =
 * thread-block cluster size (0 = no clusters: split records merged through
 * the workspace; >= 2 = the CTAs of a cluster share the stream's stages
 * dynamically and merge through distributed shared memory), out[3] =
 * clusters per (b, kv head, head group).  turbo != 0 for fkv_decode_turbo.
 * The cluster mode is opt-in: FKV_CLUSTER=1 in the environment enables it
 * for small jobs (it measured slower than the flat split on B200). */
int fkv_decode_plan(const FkvDecodeShape* s, const uint8_t* far_k, int32_t turbo, int32_t* out);

/* TurboQuant far tier, scores directly on codes.  Replaces
 * TurboFoveatedHandle::operator() (csrc/foveated_attn.cpp:407-491) and kernel
 * foveated_2tier_turbo (csrc/kernels/foveated_attn.metal:559-767); the
 * q Pi^T / q S^T products the reference does with host matmuls are computed
 * on the device inside this call. */
int fkv_decode_turbo(const FkvDecodeShape* s, const uint16_t* near_k, const uint16_t* near_v,
                     const int32_t* near_valid, const uint8_t* k_idx, const uint8_t* k_signs,
                     const uint16_t* k_norm, const uint16_t* k_gamma, const uint8_t* v_packed,
                     const uint16_t* v_scale, const float* Pi, const float* Smat,
                     const float* centroids, const uint16_t* q, const uint16_t* dec_k,
                     const uint16_t* dec_v, uint16_t* out, int32_t* flags, int32_t* tokens,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Same as fkv_decode_fp8, but allocation-free for callers that cannot call
 * cudaMalloc on their decode path (a pre-planned memory pool owned by a
 * serving runtime, a plugin host that only lends out its own tensors).  No
 * counterpart in the reference (its Metal path has no caller workspace).
 * The split scratch is a fixed 16 MiB device array inside libfkv.so, held by
 * every GPU that loads the library until exit; shapes needing more (see
 * fkv_decode_workspace_bytes) are rejected with FKV_ERR_INVALID.  The first
 * call in a CUDA context looks up the array's address in that context, so
 * make that first call before any stream capture.  All calls share the array
 * (it keeps the last call's contents; each call zeroes its status word and
 * the counters it needs): calls that overlap on the GPU race.  A shape is
 * accepted exactly when its scratch fits for both q.K paths;
 * fkv_decode_workspace_bytes(s) <= 16 MiB is sufficient for that but not
 * necessary. */
int fkv_decode_fp8_noalloc(const FkvDecodeShape* s, const uint16_t* near_k,
                           const uint16_t* near_v, const int32_t* near_valid,
                           const uint8_t* far_k, const uint8_t* far_v, const uint16_t* v_scale,
                           const uint16_t* v_zero, const uint16_t* q, const uint16_t* dec_k,
                           const uint16_t* dec_v, uint16_t* out, int32_t* flags,
                           int32_t* tokens, void* stream);

/* Status word of the last fkv_decode_fp8_noalloc call in the current
 * context (read before the next call clears it); same meaning as
 * fkv_decode_status.  No counterpart in the reference. */
int fkv_decode_noalloc_status(int32_t* status, void* stream);

/* Sequence-split variant (no reference counterpart; the reference has no
 * multi-device code): same attention over this shard's tiers, but instead of
 * the final output writes one partial record per (b, q head):
 *   part (B*Hq, D+4) f32 (16-byte aligned) = [m, l, min_near, max_far, o[0..D)] with o
 *   unnormalised (sum of exp(s-m) v);  part_arg (B*Hq) int32 = argmax far
 *   index + far_index_offset (global far index), or -1. */
int fkv_decode_fp8_partial(const FkvDecodeShape* s, const uint16_t* near_k,
                           const uint16_t* near_v, const int32_t* near_valid,
                           const uint8_t* far_k, const uint8_t* far_v, const uint16_t* v_scale,
                           const uint16_t* v_zero, const uint16_t* q, const uint16_t* dec_k,
                           const uint16_t* dec_v, int32_t far_index_offset, float* part,
                           int32_t* part_arg, void* workspace, size_t workspace_bytes,
                           void* stream);

/* Merge P shards' partial records (P, N, D+4) / (P, N) in shard order: output
 * (N, D) fp16, flags and tokens (N) int32 (earliest shard wins max_far ties). */
int fkv_combine_partials(int32_t P, int32_t N, int32_t D, const float* parts,
                         const int32_t* part_args, float spike_margin, uint16_t* out,
                         int32_t* flags, int32_t* tokens, void* stream);

/* Same merge reading each shard's block in place (no counterpart in the
 * reference): shard k's records start at parts + k * part_rank_stride and its
 * argmax values at part_args + k * arg_rank_stride (element strides, at
 * least N * (D+4) and N).  Lets a caller gather every shard's [records |
 * argmax] buffer with one collective and merge it without repacking. */
int fkv_combine_partials_strided(int32_t P, int32_t N, int32_t D, const float* parts,
                                 int64_t part_rank_stride, const int32_t* part_args,
                                 int64_t arg_rank_stride, float spike_margin, uint16_t* out,
                                 int32_t* flags, int32_t* tokens, void* stream);

/* Sequence-split exchange over peer memory (no counterpart in the reference,
 * which has no multi-device code).  Replaces the all-gather + merge of a
 * sequence-split step with one launch per rank that stores this rank's
 * [records | argmax] block (fkv_decode_fp8_partial's layout, padded to
 * fkv_exchange_block_stride floats, 16-byte aligned) into slot `rank` of
 * every rank's receive buffer with plain peer stores, each word tagged with
 * the step's sequence number in one 8-byte store, polls (bounded) its own
 * buffer until every rank's rows carry the tag, and merges the P records of
 * each row in rank order, exactly as fkv_combine_partials.
 *   peer_recv  device array of P receive-buffer addresses (own included),
 *              each fkv_exchange_recv_bytes long, zero-filled once, 64-byte
 *              aligned; peers' buffers mapped with fkv_ipc_open
 *   state      4 int32 of this rank, zero-filled once: sequence number, a
 *              block counter, unused, status (FKV_ERR_TIMEOUT if a peer's
 *              rows did not arrive in under a second)
 * At most 8 ranks.
 * Every rank must issue the same sequence of calls; one rank per GPU.
 * The receive buffers alternate between two halves by step parity. */
size_t fkv_exchange_recv_bytes(int32_t P, int32_t N, int32_t D);
int64_t fkv_exchange_block_stride(int32_t N, int32_t D);
int fkv_exchange_combine(int32_t P, int32_t rank, int32_t N, int32_t D, const float* local_block,
                         const uint64_t* peer_recv, void* my_recv, int32_t* state,
                         float spike_margin, uint16_t* out, int32_t* flags, int32_t* tokens,
                         void* stream);

/* CUDA IPC of a device buffer (no counterpart in the reference): the
 * handle (fkv_ipc_handle_bytes bytes) names the allocation holding dev_ptr,
 * and *offset is dev_ptr's offset in it; fkv_ipc_open maps it in another
 * process (peer access over NVLink) and returns the same offset into it. */
int fkv_ipc_handle_bytes(void);
int fkv_ipc_get_handle(const void* dev_ptr, uint8_t* handle, int64_t* offset);
int fkv_ipc_open(const uint8_t* handle, int64_t offset, void** dev_ptr);
int fkv_ipc_close(void* dev_ptr, int64_t offset);

/* ------------------------------------------------------------------------ */
/* Spike drain + promotion                                                  */
/* ------------------------------------------------------------------------ */

/* Opaque pipeline handle.  Replaces foveated::PromotionPipeline
 * (csrc/promotion_pipeline.h:75-141, csrc/promotion_pipeline.cpp:20-248) and
 * its binding (csrc/bindings.cpp:42-100).  One worker std::thread per
 * pipeline takes every queued promotion at once, packs the exact fp16 rows
 * from the host archive (mmapped file or pinned memory) into pinned staging,
 * moves the batch with one cudaMemcpyAsync on its own stream and scatters it
 * into near-tier headroom with a kernel, then (stream-ordered, in a second
 * kernel) stores the new near_valid[b,h] counts. */
typedef struct FkvPromo FkvPromo;

FkvPromo* fkv_promo_create(int32_t n_layers, int32_t cooldown_steps, int32_t max_per_drain,
                           int32_t device);
/* Disk archive (H_kv, S_arc, D) fp16 per file and batch row, B files packed
 * back to back = (B, H_kv, S_arc, D); archive_idx (B, H_kv, S_arc) positions. */
int fkv_promo_register_archive(FkvPromo* p, int32_t layer, const char* path_k,
                               const char* path_v, int32_t B, int32_t H_kv, int32_t S_arc,
                               int32_t D, const int32_t* archive_idx, int64_t archive_idx_len);
/* Host-memory archive (pinned or pageable), same layout; memory owned by caller. */
int fkv_promo_register_archive_host(FkvPromo* p, int32_t layer, const uint16_t* host_k,
                                    const uint16_t* host_v, int32_t B, int32_t H_kv,
                                    int32_t S_arc, int32_t D, const int32_t* archive_idx,
                                    int64_t archive_idx_len);
/* Near-tier write target of one layer: device near_k/near_v (B,H_kv,Np,D) and
 * near_valid (B,H_kv) int32; the pipeline reads near_valid once here and
 * keeps a host shadow (it is the only writer afterwards). */
int fkv_promo_register_blob(FkvPromo* p, int32_t layer, uint16_t* near_k, uint16_t* near_v,
                            int32_t* near_valid, int32_t B, int32_t H_kv, int32_t n_near_alloc,
                            int32_t D);
/* Filter one layer's spikes (host copies of flags/tokens (B,Hq), far_idx
 * (B,H_kv,F)) and queue promotions.  Returns the number queued (>= 0). */
int fkv_promo_drain(FkvPromo* p, int32_t layer, const int32_t* flags, const int32_t* tokens,
                    const int32_t* far_idx, int32_t B, int32_t Hq, int32_t H_kv, int32_t n_far,
                    int32_t step);
/* Block until queued promotions are issued, then make `stream` wait for them
 * (deterministic mode).  timeout_ms bounds the host wait. */
int fkv_promo_flush(FkvPromo* p, void* stream, int32_t timeout_ms);
/* stats[6] = detected, queued, deduplicated, cooled_down, completed, headroom_full */
int fkv_promo_stats(FkvPromo* p, uint64_t* stats);
int fkv_promo_stop(FkvPromo* p);
void fkv_promo_destroy(FkvPromo* p);

#ifdef __cplusplus
}
#endif
#endif /* FKV_H_ */
