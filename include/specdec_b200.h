/*
 * specdec_b200.h -- C ABI of the B200 (sm_100a) decode / speculative-verify hot path.
 *
 * Every entry point takes plain device pointers, element strides and sizes, a
 * caller-owned workspace and a cudaStream_t (passed as void*), launches on that
 * stream, allocates nothing, never synchronises the device and returns a status
 * code (SDB_OK or one of SDB_ERR_*), so every call can be captured in a CUDA
 * graph.  Tensor layouts are the reference's (henry-tmp-de/specdec-nanovllm).
 *
 * Thread safety: calls are re-entrant across streams as long as concurrent calls
 * use distinct workspaces.
 */
#ifndef SPECDEC_B200_H
#define SPECDEC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define SDB_OK                 0
#define SDB_ERR_INVALID_ARG    1   /* null pointer, negative size, bad stride      */
#define SDB_ERR_UNSUPPORTED    2   /* shape / dtype combination not built          */
#define SDB_ERR_WORKSPACE      3   /* workspace missing or too small               */
#define SDB_ERR_CUDA           4   /* launch or driver error (see sdb_last_error)  */

/* Bits a kernel ORs into the workspace error word (sdb_*_error_word). */
#define SDB_KERR_SEQLEN        0x1 /* cache length < 0 or > max_blocks * page      */
#define SDB_KERR_BLOCK_ID      0x2 /* block table entry outside [0, num_blocks)    */
#define SDB_KERR_TIMEOUT       0x4 /* a bounded wait gave up                       */
#define SDB_KERR_TOKEN         0x8 /* draft token outside [0, vocab)               */
#define SDB_KERR_SLOT          0x10 /* fused store: slot differs from the position's */

/* ---- dtypes --------------------------------------------------------------- */
#define SDB_F32   0
#define SDB_BF16  1
#define SDB_F16   2

/* Human-readable message of the last SDB_ERR_CUDA on this thread. */
const char* sdb_last_error(void);

/* Library build identity: "sm_100a" and the list of kernels compiled in. */
const char* sdb_build_info(void);

/* =========================================================================
 * Paged decode / verify attention.
 *
 * Replaces, with one kernel family:
 *   - flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens, block_table,
 *     softmax_scale, causal=True)           nanovllm/layers/attention.py:78-81 (decode, n_q = 1)
 *   - flash_attn_varlen_func(q, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k, ...,
 *     causal=True, block_table)              nanovllm/layers/attention.py:67-70 (verify, n_q = k+1)
 *   - paged_decode_attention / paged_decode_attention_cuda
 *                                            nanovllm/kernels/paged_decode_attn.py:352,
 *                                            nanovllm/kernels/paged_decode_attn_cuda.py:52
 *
 *   q       (B*n_q, Hq, D)          rows b*n_q .. b*n_q+n_q-1 belong to sequence b
 *   k_cache (num_blocks, page, Hkv, D)  the nano-vllm / flash-attn paged layout
 *   v_cache same layout (may alias a different base with the same strides)
 *   block_tables (B, max_blocks) int32, -1 padded; only the first ceil(L/page)
 *                entries of a row are read
 *   cache_seqlens (B) int32 L_b: keys in the cache, the n_q new ones included
 *   out     (B*n_q, Hq, D)          same dtype as q
 *
 * Row r (0..n_q-1) of sequence b attends to keys j <= L_b - n_q + r (flash-attn's
 * bottom-right causal alignment); rows that see no key, and every row of an
 * L_b = 0 sequence, are written as zeros.  Strides are in elements; the last dim
 * of q / out / caches must be contiguous.
 *
 * dtype: SDB_BF16 / SDB_F16 (tensor-core path: D = 128, page % 64 == 0,
 *        n_q*Hq/Hkv <= 64) or SDB_F32 (CUDA-core path, fp32 accumulate, any
 *        page, D in {32, 64, 128, 256}, n_q*Hq/Hkv <= 64).  B * Hkv <= 65536.
 * splits: partial slots per (sequence, kv head) the workspace is sized for; 0
 *         picks sdb_paged_attention_default_splits().  The decomposition is chosen
 *         from the static shape (max_blocks * page), never from device data: with
 *         16-bit KV, D = 128, page % 128 == 0 and n_q*Hq/Hkv <= 32 (tcgen05 kernel)
 *         either every pair is split into `splits` key chunks, or -- when the
 *         shape plan prefers it and `splits` covers it -- a balanced partition of
 *         all keys over groups of CTAs that splits only pairs cut by a group
 *         boundary; on the other paths `splits` is the key-chunk count.
 * workspace: sdb_paged_attention_workspace_size() bytes, 256-byte aligned,
 *         zero-filled once before first use (the kernels leave it re-usable).
 * ========================================================================= */
size_t sdb_paged_attention_workspace_size(int B, int n_q, int Hq, int Hkv, int D, int splits);

int sdb_paged_attention_default_splits(int B, int n_q, int Hq, int Hkv, int D, int page,
                                       int max_blocks, int dtype);

/* The decomposition sdb_paged_attention launches for this static shape and `splits`
 * (0 = default), without launching: *kernel receives one of SDB_ATTN_PLAN_* (-1 for
 * invalid sizes), *slots the partial slots per (sequence, kv head) the launch uses (the
 * strided split count, or the slots of the grouped partition); returns the workspace
 * bytes that launch needs (0 for invalid sizes).  Follows the same kernel choice as the
 * launch (SDB_ATTN_KERNEL=mma included).  Host only: no CUDA call beyond the SM count.
 * The reference has no counterpart (its split count is a call argument,
 * nanovllm/kernels/paged_decode_attn_cuda.py:52). */
#define SDB_ATTN_PLAN_CUDA_CORE        0  /* fp32 / other shapes: one CTA per (kv head, seq) */
#define SDB_ATTN_PLAN_MMA              1  /* mma.sync kernel, `slots` key chunks per pair    */
#define SDB_ATTN_PLAN_TCGEN05_STRIDED  2  /* tcgen05 kernel, `slots` key chunks per pair     */
#define SDB_ATTN_PLAN_TCGEN05_GROUPED  3  /* tcgen05 kernel, balanced partition over groups  */
size_t sdb_paged_attention_plan(int B, int n_q, int Hq, int Hkv, int D, int page, int max_blocks,
                                int dtype, int splits, int* kernel, int* slots);

int sdb_paged_attention(const void* q, int64_t q_stride_row, int64_t q_stride_head,
                        const void* k_cache, const void* v_cache,
                        int64_t kv_stride_block, int64_t kv_stride_page, int64_t kv_stride_head,
                        const int32_t* block_tables, int64_t bt_stride,
                        const int32_t* cache_seqlens,
                        void* out, int64_t o_stride_row, int64_t o_stride_head,
                        int B, int n_q, int Hq, int Hkv, int D, int page,
                        int max_blocks, int num_blocks,
                        float softmax_scale, int dtype, int splits,
                        void* workspace, size_t workspace_bytes, void* stream);

/* No-allocation variant of sdb_paged_attention (no counterpart in the reference).
 * For callers that cannot allocate device memory when they run attention -- a
 * plugin inside another runtime's enqueue callback whose memory pool forbids raw
 * allocations, a steady-state serving loop that cannot afford cudaMalloc's
 * implicit device-wide synchronisation, a deployment with a fixed memory budget.
 * Same arguments as sdb_paged_attention without the workspace: the split
 * partials and merge counters live in a file-scope device array of
 * SDB_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until the
 * process exits.  Shapes needing more scratch (sized for the split count the launch
 * actually uses, see sdb_paged_attention_plan) return SDB_ERR_WORKSPACE before any
 * launch.  The first call on a device (that device current) looks the array up and
 * clears its error word and counters with cudaMemsetAsync on the given stream; that
 * first call must not be made while the stream is being captured into a CUDA graph
 * (it returns SDB_ERR_INVALID_ARG if it is).  All calls share the array: calls that
 * overlap on the GPU race and must be serialised by the caller.  Allocates nothing. */
#define SDB_NOALLOC_SCRATCH_BYTES (16u << 20)
int sdb_paged_attention_noalloc(const void* q, int64_t q_stride_row, int64_t q_stride_head,
                                const void* k_cache, const void* v_cache,
                                int64_t kv_stride_block, int64_t kv_stride_page, int64_t kv_stride_head,
                                const int32_t* block_tables, int64_t bt_stride,
                                const int32_t* cache_seqlens,
                                void* out, int64_t o_stride_row, int64_t o_stride_head,
                                int B, int n_q, int Hq, int Hkv, int D, int page,
                                int max_blocks, int num_blocks,
                                float softmax_scale, int dtype, int splits, void* stream);

/* The error word of sdb_paged_attention_noalloc on the current device (no counterpart
 * in the reference).  Those callers have no workspace, so this is how they see the
 * SDB_KERR_* bits the kernels record (a clamped block id, a clamped cache length, a
 * bounded wait that gave up).  Enqueues on `stream` a 4-byte copy of the word into
 * *host_word (valid once the stream has synchronised; pinned or pageable memory)
 * and, with clear != 0, then resets the word to 0.  The bits otherwise accumulate
 * over every call on the device.  Allocates nothing. */
int sdb_paged_attention_noalloc_error_word(int32_t* host_word, int clear, void* stream);

/* Memory-floor twin of sdb_paged_attention: the same grid, the same TMA loads
 * of every visible K/V tile, no math; writes one checksum word per CTA into the
 * workspace.  Reference counterpart: paged_decode_readonly_kernel,
 * nanovllm/kernels/paged_decode_attn_cuda.cu:654-705. */
int sdb_paged_attention_readonly(const void* q, int64_t q_stride_row, int64_t q_stride_head,
                                 const void* k_cache, const void* v_cache,
                                 int64_t kv_stride_block, int64_t kv_stride_page,
                                 int64_t kv_stride_head,
                                 const int32_t* block_tables, int64_t bt_stride,
                                 const int32_t* cache_seqlens,
                                 int B, int n_q, int Hq, int Hkv, int D, int page,
                                 int max_blocks, int num_blocks, int dtype, int splits,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* Error word the attention kernels OR SDB_KERR_* bits into (device pointer
 * inside the workspace; read it after a synchronise when debugging). */
const int32_t* sdb_paged_attention_error_word(const void* workspace, int B, int n_q, int Hq,
                                              int Hkv, int D, int splits);


/* store_kvcache: scatter the new K/V rows of this step into the paged cache.
 * Replaces store_kvcache / store_kvcache_kernel   nanovllm/layers/attention.py:10-40.
 *   key, value (N, Hkv, D); slot_mapping (N) int32, slot = block * page + offset,
 *   -1 = skip the row (graph padding).  workspace: the attention workspace (its
 *   error word records slots past num_blocks). */
int sdb_store_kvcache(const void* key, int64_t key_stride_tok, int64_t key_stride_head,
                      const void* value, int64_t value_stride_tok, int64_t value_stride_head,
                      void* k_cache, void* v_cache,
                      int64_t kv_stride_block, int64_t kv_stride_page, int64_t kv_stride_head,
                      const int32_t* slot_mapping, int N, int Hkv, int D, int page, int num_blocks,
                      int dtype, void* workspace, void* stream);

/* Fused store + attention: the step's new K / V rows go into the paged cache and
 * the queries attend over it, in one call.  The result equals sdb_store_kvcache
 * (key, value, ..., slot_mapping, N = B * n_q) followed by sdb_paged_attention
 * with the remaining arguments.
 * Replaces the store_kvcache + attention pair of Attention.forward
 *                                           nanovllm/layers/attention.py:59-81.
 *   key, value   (B*n_q, Hkv, D): row b*n_q + i is new token i of sequence b, at
 *                cache position cache_seqlens[b] - n_q + i (strides in elements)
 *   slot_mapping (B*n_q) int32: -1 (skip the row) or the slot the block table
 *                gives that position (nanovllm/engine/model_runner.py:469-476
 *                for decode, :537-548 for verify)
 * On the tcgen05 path the attention kernel writes the rows itself: the CTA whose
 * key range holds a row's position writes it just before the TMA load of that
 * tile, so the row costs no extra launch and no second read.  A slot that is
 * neither -1 nor the position's own slot is still written and sets SDB_KERR_SLOT
 * (the attention then reads the position's own slot, as a separate store
 * followed by attention would).  The other paths launch the store kernel and
 * then attention.  No other sequence's block table may name a block that
 * receives a new row in the same call (the reference's tail blocks are private). */
int sdb_paged_attention_store(const void* q, int64_t q_stride_row, int64_t q_stride_head,
                              const void* key, int64_t key_stride_tok, int64_t key_stride_head,
                              const void* value, int64_t value_stride_tok, int64_t value_stride_head,
                              const int32_t* slot_mapping,
                              void* k_cache, void* v_cache,
                              int64_t kv_stride_block, int64_t kv_stride_page, int64_t kv_stride_head,
                              const int32_t* block_tables, int64_t bt_stride,
                              const int32_t* cache_seqlens,
                              void* out, int64_t o_stride_row, int64_t o_stride_head,
                              int B, int n_q, int Hq, int Hkv, int D, int page,
                              int max_blocks, int num_blocks,
                              float softmax_scale, int dtype, int splits,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Attention prologue of a Qwen3 layer in one launch: split of the fused QKV
 * projection output, per-head RMSNorm of q and k, rotary embedding of q and k,
 * and the store of the step's k / v rows into the paged cache.
 * Replaces Qwen3Attention.forward :78-85 (split, q_norm, k_norm, rotary_emb)
 *   nanovllm/models/qwen3.py:77-86, RMSNorm.rms_forward nanovllm/layers/layernorm.py:16-25,
 *   RotaryEmbedding.forward / apply_rotary_emb nanovllm/layers/rotary_embedding.py:6-14, 38-50,
 * and the store_kvcache of Attention.forward (attention.py:59-63).
 *   qkv           (T, (Hq + 2 Hkv) D) rows qkv_stride_tok apart: q heads, k heads, v heads
 *   q_norm_weight, k_norm_weight  (D) in the model dtype, or NULL (models with a qkv
 *                 bias have no q/k norm, qwen3.py:68-70)
 *   cos_sin_cache (max_position, D) float32 rows cos_sin_stride_pos apart,
 *                 [cos(D/2) | sin(D/2)] (the RotaryEmbedding buffer)
 *   positions     (T) int64
 *   q_out         (T, Hq, D) normalised and rotated q
 *   k_out, v_out  NULL or (T, Hkv, D): the normalised, rotated k and the v rows
 *   k_cache, v_cache, slot_mapping: the paged caches and (T) int32 slots (-1 skips a
 *                 row); slot_mapping NULL stores nothing
 * Numerics follow the reference's eager torch: RMSNorm in float32 with 1/sqrt, the
 * normalised value rounded to the model dtype before the weight multiply; rotary
 * products and sums rounded separately, then rounded to the model dtype.
 * dtype: SDB_BF16 / SDB_F16 / SDB_F32; D in {64, 128, 256}.  workspace: the
 * attention workspace (its error word records slots past num_blocks and positions
 * outside [0, max_position)). */
int sdb_qk_norm_rope_store(const void* qkv, int64_t qkv_stride_tok,
                           const void* q_norm_weight, const void* k_norm_weight, float eps,
                           const float* cos_sin_cache, int64_t cos_sin_stride_pos, int max_position,
                           const int64_t* positions,
                           void* q_out, int64_t q_stride_tok, int64_t q_stride_head,
                           void* k_out, void* v_out, int64_t kv_stride_tok, int64_t kv_stride_head,
                           void* k_cache, void* v_cache,
                           int64_t kv_stride_block, int64_t kv_stride_page, int64_t kv_stride_head_cache,
                           const int32_t* slot_mapping,
                           int T, int Hq, int Hkv, int D, int page, int num_blocks,
                           int dtype, void* workspace, void* stream);

/* =========================================================================
 * verify_batch: lossless rejection sampling of k drafted tokens.
 *
 * Replaces verify_batch(draft_probs, target_logits, draft_tokens, temperatures,
 * draft_is_point_mass) -> VerifyResult      nanovllm/spec_decode/verify.py:42-175
 *
 *   draft_logits  (B, k, V) float32  raw draft logits (or probabilities when
 *                 draft_is_point_mass != 0, used as-is, verify.py:86-87)
 *   target_logits (B, target_rows, V) float32, target_rows = k+1 (or k)
 *   draft_tokens  (B, k) int64
 *   temperatures  (B) float32 or NULL (no division)
 *   uniforms      (B, k) float32 or NULL: acceptance draws; NULL -> Philox
 *                 stream 0 keyed by (seed, offset)
 *   exponentials  (B, V) float32 or NULL: bonus Exp(1) draws; NULL -> Philox
 *                 stream 1 keyed by (seed, offset)
 *   out_accepted  (B) int64, out_bonus (B) int64, out_accept_mask (B, k) uint8
 *   workspace     sdb_verify_workspace_size() bytes, zero-filled once.
 * ========================================================================= */
size_t sdb_verify_workspace_size(int B, int k, int target_rows, int V);

int sdb_verify_batch(const float* draft_logits, const float* target_logits,
                     const int64_t* draft_tokens, const float* temperatures,
                     const float* uniforms, const float* exponentials,
                     uint64_t seed, uint64_t offset, int draft_is_point_mass,
                     int64_t* out_accepted, int64_t* out_bonus, uint8_t* out_accept_mask,
                     int B, int k, int target_rows, int V,
                     void* workspace, size_t workspace_bytes, void* stream);

/* verify_batch with logits of any float type, read as float32 exactly in the kernels
 * (the reference converts with .float(), verify.py:194): the engine passes the
 * LM head's bf16 target logits straight in (model_runner.py:1101-1103), so no
 * (B, k+1, V) float32 copy is made.  draft_dtype / target_dtype: SDB_F32,
 * SDB_BF16 or SDB_F16; everything else as sdb_verify_batch (which is this call
 * with both SDB_F32). */
int sdb_verify_batch_ex(const void* draft_logits, int draft_dtype,
                        const void* target_logits, int target_dtype,
                        const int64_t* draft_tokens, const float* temperatures,
                        const float* uniforms, const float* exponentials,
                        uint64_t seed, uint64_t offset, int draft_is_point_mass,
                        int64_t* out_accepted, int64_t* out_bonus, uint8_t* out_accept_mask,
                        int B, int k, int target_rows, int V,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Graph-safe form of sdb_verify_batch_ex (draws generated in-kernel): the Philox offset is
 * read from device memory (*offset_dev, 8-byte aligned) when the kernels run and advanced
 * by one after the call (a one-thread launch on the same stream), so a call captured in
 * a CUDA graph draws new values on every replay.  The draws of a call that finds
 * *offset_dev == v equal those of sdb_verify_batch_ex with offset v.  The reference
 * draws with torch's generator inside the call (verify.py:120, :209); its eager calls
 * advance it on every call, which a host-side offset captured in a graph would not. */
int sdb_verify_batch_dev_offset(const void* draft_logits, int draft_dtype,
                                const void* target_logits, int target_dtype,
                                const int64_t* draft_tokens, const float* temperatures,
                                uint64_t seed, uint64_t* offset_dev, int draft_is_point_mass,
                                int64_t* out_accepted, int64_t* out_bonus, uint8_t* out_accept_mask,
                                int B, int k, int target_rows, int V,
                                void* workspace, size_t workspace_bytes, void* stream);

/* verify_batch over vocabulary shards: the LM head split by columns across tp ranks
 * (ParallelLMHead, nanovllm/layers/embed_head.py:56-75).  The reference gathers the
 * full logits on rank 0 (:71-74); here every rank keeps its shard and the ranks
 * exchange per-sequence statistics only.  Four phases; between phases the caller
 * all-gathers each rank's `send` buffer (sdb_verify_shard_send_floats(B, k,
 * target_rows, phase) floats) into `gathered` in rank order (tp x that many):
 *   1: local statistics; send = per sequence each row's (max, sum exp) and the
 *      candidates' logits on the rank that owns their columns (NaN elsewhere)
 *   2: the decisions from the gathered summaries (out_accepted, out_accept_mask),
 *      then this rank's residual / p sums of row `accepted`; send = those sums
 *   3: this rank's bonus argmax under the global normaliser; send = (best value,
 *      global column as float bits)
 *   4: out_bonus from the gathered bests
 * Draws are keyed by global columns (the single-device streams).  Every rank ends
 * with identical outputs, equal to sdb_verify_batch_ex on the full logits except
 * where two values tie within float32 rounding (the shards' sums are added in another
 * order).  vocab_start: this rank's first column; V_local its column count; the
 * workspace (sdb_verify_workspace_size(B, k, target_rows, V_local)) carries the
 * decisions from phase 2 to phases 3-4: keep it between the phases of one call. */
size_t sdb_verify_shard_send_floats(int B, int k, int target_rows, int phase);
int sdb_verify_batch_shard(int phase, const void* draft_logits, int draft_dtype,
                           const void* target_logits, int target_dtype,
                           const int64_t* draft_tokens, const float* temperatures,
                           const float* uniforms, const float* exponentials,
                           uint64_t seed, uint64_t offset, int draft_is_point_mass,
                           int64_t* out_accepted, int64_t* out_bonus, uint8_t* out_accept_mask,
                           int B, int k, int target_rows, int V_local, int vocab_start, int V_total,
                           int tp, const float* gathered, float* send,
                           void* workspace, size_t workspace_bytes, void* stream);

/* Philox streams of the samplers written out (test and debugging aid): stream 0
 * as uniforms [rows, cols], stream 1 (verify_batch) or 2 (sample) as
 * exponentials [rows, cols]. */
int sdb_philox_fill(float* out, int rows, int cols, uint64_t seed, uint64_t offset,
                    int stream_id, void* stream);

/* =========================================================================
 * sample: Gumbel-max token sampling with exponential noise.
 *
 * Replaces Sampler.forward(logits, temperatures)   nanovllm/layers/sampler.py:8-12
 * and the draft step's sampling + logits copy   nanovllm/spec_decode/draft_proposer.py:505-510
 *   tokens[b] = argmax_i softmax(logits[b] / T[b])_i / max(E[b, i], 1e-10),  E ~ Exp(1),
 *   first index on ties (torch.argmax).
 *
 *   logits       (B, V) f32 / bf16 / f16 (dtype), rows logits_stride_row elements
 *                apart, contiguous within a row; converted to float32 exactly
 *   temperatures (B) float32 or NULL (no division); T > 0 as in the reference
 *   exponentials (B, V) float32 or NULL: the noise; NULL -> Philox stream 2 keyed
 *                by (seed, offset), E = -log(U) (sdb_philox_fill, stream_id 2)
 *   tokens       int64, row b's token at tokens[b * tokens_stride]
 *   logits_f32   NULL, or (B, V) float32 rows logits_f32_stride_row apart that
 *                receive logits converted to float32 (the draft step's copy)
 * workspace: sdb_sample_workspace_size(B, V) bytes, 256-byte aligned (no zeroing
 * needed).  Two launches (the second a programmatic dependent launch); one read of
 * the logits.  The inputs are not modified (the reference divides fp32 logits in
 * place).
 * ========================================================================= */
size_t sdb_sample_workspace_size(int B, int V);

/* Graph-safe form of sdb_sample with in-kernel noise: the Philox offset is read from
 * device memory (*offset_dev, 8-byte aligned) when the kernels run and advanced by one
 * after the call, so a captured call samples new noise on every replay (the reference's
 * exponential_() advances torch's generator, sampler.py:11, draft_proposer.py:508).  A
 * call that finds *offset_dev == v samples what sdb_sample does with offset v. */
int sdb_sample_dev_offset(const void* logits, int64_t logits_stride_row, int dtype,
                          const float* temperatures, uint64_t seed, uint64_t* offset_dev,
                          int64_t* tokens, int64_t tokens_stride,
                          float* logits_f32, int64_t logits_f32_stride_row,
                          int B, int V, void* workspace, size_t workspace_bytes, void* stream);
int sdb_sample(const void* logits, int64_t logits_stride_row, int dtype,
               const float* temperatures, const float* exponentials,
               uint64_t seed, uint64_t offset,
               int64_t* tokens, int64_t tokens_stride,
               float* logits_f32, int64_t logits_f32_stride_row,
               int B, int V, void* workspace, size_t workspace_bytes, void* stream);

/* =========================================================================
 * W8A16 linear: y = x @ (q * scale)^T (+ bias), int8 weights dequantised in
 * registers.
 *
 * Replaces int8_linear(x, qweight, scale, bias, granularity, group_size)
 *                                           nanovllm/layers/quant.py:262-310
 *
 *   x     (M, K) act_dtype (SDB_BF16 or SDB_F16), rows contiguous, x_stride_row
 *   qweight (N, K) int8 row-major (K contiguous)
 *   scale (N) per output channel (group_size == 0) or (N, K/group_size),
 *         scale_dtype SDB_BF16 / SDB_F16 / SDB_F32
 *   bias  (N) act_dtype or NULL
 *   y     (M, N) act_dtype, y_stride_row
 *   Requires K % 64 == 0; group_size 0 or a multiple of 64 dividing K.
 *   workspace: sdb_w8a16_workspace_size() bytes (split-K partials), zero-filled once.
 *   Kernels: mma.sync up to 16 tokens and for grouped scales; with per-channel scales
 *   and K % 128 == 0, tcgen05 above (17-128 tokens: split-K across a thread-block
 *   cluster where that plan is balanced, else stream-K over persistent CTAs; more
 *   than 128 tokens: stream-K in token blocks of at most 256).
 * ========================================================================= */
size_t sdb_w8a16_workspace_size(int M, int N, int K);

int sdb_w8a16_linear(const void* x, int64_t x_stride_row, const int8_t* qweight,
                     const void* scale, int scale_dtype, int group_size,
                     const void* bias, void* y, int64_t y_stride_row,
                     int M, int N, int K, int act_dtype,
                     void* workspace, size_t workspace_bytes, void* stream);

/* quantize_weight: symmetric int8 quantisation of a (N, K) weight.
 * Replaces quantize_weight(w, granularity, group_size)  nanovllm/layers/quant.py:123-148.
 * w float32/bf16/f16 (w_dtype), q out int8 (N, K), scale out (N) or (N, K/G) in
 * scale_dtype (the scale is computed in float32 and rounded once, as the reference). */
int sdb_quantize_weight(const void* w, int w_dtype, int8_t* q, void* scale, int scale_dtype,
                        int N, int K, int group_size, void* stream);

/* =========================================================================
 * Decoder-layer elementwise steps (model side of the end-to-end step).
 *
 * sdb_rms_norm replaces RMSNorm.rms_forward / add_rms_forward
 *                                           nanovllm/layers/layernorm.py:17-43
 *   s = x (+ residual_in) in float32; residual_out (may be NULL) = s rounded to dtype;
 *   out = (s * rsqrt(mean(s^2) + eps)) rounded to dtype, times weight, rounded.
 *   x, residual_in, out, residual_out (T, H) rows *_stride elements apart (16-byte aligned
 *   rows; out may alias x and residual_out residual_in), weight (H); H % 8 == 0, H <= 8192.
 * sdb_silu_mul replaces SiluAndMul.forward  nanovllm/layers/activation.py:8-13
 *   gate_up (T, 2F) rows [gate | up], out (T, F) = silu(gate) * up, silu rounded to dtype
 *   before the product as torch rounds it; F % 8 == 0.
 * dtype: SDB_BF16 or SDB_F16.
 * ========================================================================= */
int sdb_rms_norm(const void* x, int64_t x_stride, const void* residual_in, int64_t residual_in_stride,
                 void* out, int64_t out_stride, void* residual_out, int64_t residual_out_stride,
                 const void* weight, int T, int H, float eps, int dtype, void* stream);

int sdb_silu_mul(const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride,
                 int T, int F, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPECDEC_B200_H */
