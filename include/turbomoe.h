/*
 * turbomoe.h -- C ABI of libturbomoe.so, the B200 (sm_100a) kernels behind the
 * FP8 mixture-of-experts hot path of Turbo-LLM (router + expert FFN).
 *
 * Conventions
 *   - Every pointer argument is DEVICE memory unless stated otherwise.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Every entry point returns 0 (TM_OK) on success or a negative TM_ERR_*
 *     code; tm_last_error() returns a thread-local message for the last failure.
 *     Argument errors are reported before anything is launched.
 *   - The library never allocates on these paths.  The caller owns every buffer,
 *     including one workspace per stream sized by tm_workspace_bytes() and
 *     zeroed once by tm_workspace_init().  Kernels keep the workspace's
 *     counters self-resetting, so consecutive calls (and CUDA-graph replays)
 *     need no further initialisation.  Calls that share a workspace must be
 *     ordered on one stream.
 *   - Activations ("act") are fp32, fp16 or bf16 (tm_dtype); expert weights are
 *     FP8 e4m3 with one fp32 `weight_scale_inv` per 128x128 block.
 *
 * Reference interfaces (kaushikharsh99/Turbo-LLM, paths inside that project):
 *   The reference is pure Python; its "plugin boundary" is the class swap in
 *   runtime/engine.py:14-21 (RouterExecutor, MoEExecutor, ExpertLoader).  The
 *   Python drop-ins in turbo-llm_b200/{execution,loader} call this ABI through
 *   ctypes; each function below names the reference code it replaces.
 */
#ifndef TURBOMOE_H
#define TURBOMOE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TM_ABI_VERSION 1

#define TM_OK 0
#define TM_ERR_INVALID (-1)     /* bad argument (null pointer, shape, dtype) */
#define TM_ERR_CUDA (-2)        /* a CUDA runtime call failed */
#define TM_ERR_WORKSPACE (-3)   /* workspace too small */
#define TM_ERR_UNSUPPORTED (-4) /* shape outside what the kernels implement */

typedef enum { TM_DTYPE_F32 = 0, TM_DTYPE_F16 = 1, TM_DTYPE_BF16 = 2 } tm_dtype;

/* Device-side status bits written into the workspace (tm_workspace_status). */
#define TM_STATUS_BAD_EXPERT_ID 1u  /* a top-k index was outside [0, n_experts) */
#define TM_STATUS_TIMEOUT 2u        /* a bounded device-side wait gave up; outputs are invalid */
#define TM_STATUS_BAD_TOKEN_ID 8u   /* a token id outside [0, vocab) or a position outside the KV cache */
#define TM_STATUS_PEER_FAILED 4u    /* expert parallelism: an owner rank gave up on this call (it timed
                                       out waiting for a source); this rank's outputs are invalid */

int tm_abi_version(void);
const char *tm_last_error(void);

/* ------------------------------------------------------------------------ */
/* K0: FP8 block dequantisation.
 * Replaces ExpertLoader.dequantize_weight (loader/expert_loader.py:127-160).
 * out[r,c] = cast(w[r,c]) * cast(scale_inv[r/128, c/128]) evaluated exactly as
 * the reference does in out_dtype: for fp32 one RN fp32 multiply; for fp16 and
 * bf16 both operands are first rounded to out_dtype, the product is formed in
 * fp32 and rounded to out_dtype (round-to-nearest-even).  rows, cols must be
 * multiples of 128.  w: uint8 e4m3 [rows, cols] row-major; scale_inv fp32
 * [rows/128, cols/128]; out [rows, cols] of out_dtype. */
int tm_dequant_fp8_block(const uint8_t *w, const float *scale_inv, int64_t rows,
                         int64_t cols, void *out, int out_dtype, void *stream);

/* ------------------------------------------------------------------------ */
/* K5: packed, device-resident expert layout (replaces the slot cache of
 * ExpertLoader.load_expert / load_expert_dynamic, loader/expert_loader.py:269-576,
 * and the RAM tier cache/ram_cache.py:6-101: every expert is uploaded once).
 *
 * Per expert (H = hidden, I = intermediate):
 *   w13: gate and up interleaved in 16-byte column chunks,
 *        [I/16][H/16][2 (gate, up)][16 rows][16 bytes]          = 2*I*H bytes
 *        (a 16-row group over all of H is one contiguous 32*H-byte tile; each
 *        16x16 chunk is one m16k16 tensor-core A tile)
 *   s13: [I/128][2][H/128] fp32                                  = 2*(I/128)*(H/128)
 *   w2 : down, [H/16][I/16][16 rows][16 bytes]                   = H*I bytes
 *   s2 : [H/128][I/128] fp32
 * Experts are stacked: expert e starts at e * tm_packed_*(...). */
int64_t tm_packed_w13_bytes(int hidden, int inter);
int64_t tm_packed_s13_floats(int hidden, int inter);
int64_t tm_packed_w2_bytes(int hidden, int inter);
int64_t tm_packed_s2_floats(int hidden, int inter);

/* Pack n_experts experts from checkpoint layout.  gate/up: [n, I, H] e4m3
 * (row-major, as <expert>.gate_proj.weight); gate_s/up_s: [n, I/128, H/128];
 * down: [n, H, I]; down_s: [n, H/128, I/128].  Outputs are the first n
 * experts of the packed arrays above.  H and I must be multiples of 128. */
int tm_pack_experts(const uint8_t *gate, const float *gate_s, const uint8_t *up,
                    const float *up_s, const uint8_t *down, const float *down_s,
                    int n_experts, int hidden, int inter, uint8_t *w13, float *s13,
                    uint8_t *w2, float *s2, void *stream);

/* Dequantise one packed expert back to dense [I,H], [I,H], [H,I] tensors of
 * out_dtype with the arithmetic of tm_dequant_fp8_block.  Backs
 * ExpertLoader.load_expert's return value (loader/expert_loader.py:362-576);
 * not on the hot path.  Any of the three outputs may be NULL. */
int tm_unpack_expert(const uint8_t *w13, const float *s13, const uint8_t *w2,
                     const float *s2, int hidden, int inter, void *gate_out,
                     void *up_out, void *down_out, int out_dtype, void *stream);

/* ------------------------------------------------------------------------ */
/* Workspace: routing plan, intermediate activations and counters for one
 * MoE layer call with at most max_tokens tokens. */
int64_t tm_workspace_bytes(int64_t max_tokens, int n_experts, int top_k, int hidden,
                           int inter, int shared_inter);
int tm_workspace_init(void *ws, int64_t ws_bytes, void *stream);
/* Copy the device status word (TM_STATUS_* bits) to *host_status and clear it;
 * synchronises `stream`. */
int tm_workspace_status(void *ws, int64_t ws_bytes, uint32_t *host_status, void *stream);
/* Byte offsets (within the workspace) of the routing plan written by
 * tm_router_topk / tm_route_plan for a call with `tokens` tokens, in this
 * order: meta (int32 [n_active, pairs, tokens]), counts (int32 [E]), offsets
 * (int32 [E+1]), act_list (int32 [n_active], ascending expert ids), slot_token
 * (int32 [T*k]), slot_pair (int32 [T*k], pair = token*k + rank), pair_slot
 * (int32 [T*k]), status (uint32).  Lets a caller inspect or reuse the plan
 * (the reference builds the same grouping implicitly in execution/moe.py:132,164). */
int tm_plan_offsets(int64_t tokens, int n_experts, int top_k, int64_t *out8);

/* ------------------------------------------------------------------------ */
/* K1: fused router.  Replaces RouterExecutor.compute_routing
 * (execution/router.py:15-42) and the implicit grouping of
 * MoEExecutor.execute_layer (execution/moe.py:132,164-165).
 *   logits = x @ router_w^T, fp32 accumulation, rounded to act dtype;
 *   p = softmax(logits) in fp32; top_k by value (ties: lower expert id first);
 *   w = p / sum(p_topk) in fp32, stored in act dtype; idx stored as int64.
 * Also writes the routing plan into the workspace: per-expert counts and
 * offsets, the list of active experts (ascending) and the stable permutation
 * (experts ascending, tokens ascending within an expert), which the expert
 * kernels consume.  x: [tokens, hidden] act; router_w: [n_experts, hidden] act;
 * topk_idx: [tokens, top_k] int64; topk_w: [tokens, top_k] act;
 * logits_out: optional [tokens, n_experts] act (NULL to skip). */
int tm_router_topk(const void *x, int64_t tokens, int hidden, int act_dtype,
                   const void *router_w, int n_experts, int top_k, int64_t *topk_idx,
                   void *topk_w, void *logits_out, void *ws, int64_t ws_bytes,
                   void *stream);
/* One token, bf16/fp16, E <= 128, top_k <= 8, hidden <= 2048: RMSNorm of x
 * (tm_rmsnorm's arithmetic, the same bits) written to x_norm_out, then
 * tm_router_topk of the normalised token, in one launch: the decode step's
 * post-attention norm fused into the router (the expert kernels then read
 * x_norm_out). */
int tm_rmsnorm_router_topk(const void *x, int hidden, int act_dtype, const void *norm_w, float eps,
                           void *x_norm_out, const void *router_w, int n_experts, int top_k, int64_t *topk_idx,
                           void *topk_w, void *logits_out, void *ws, int64_t ws_bytes, void *stream);

/* Build only the routing plan from caller-supplied top-k indices (used when
 * MoEExecutor.execute_layer receives indices that did not come from
 * tm_router_topk).  Indices outside [0, n_experts) are skipped and flagged
 * with TM_STATUS_BAD_EXPERT_ID. */
int tm_route_plan(const int64_t *topk_idx, int64_t tokens, int top_k, int n_experts,
                  void *ws, int64_t ws_bytes, void *stream);

/* ------------------------------------------------------------------------ */
/* K2: gate+up dequant-GEMV with SwiGLU for the tokens of every active expert
 * (and the shared expert when sh_w13 != NULL).  Replaces the gate/up/SiLU part
 * of moe_seq (execution/moe.py:15-17), of the multi-token loop
 * (execution/moe.py:168-172) and of the shared expert (moe.py:74-77,191-194).
 * Needs the plan of tm_router_topk / tm_route_plan in `ws`.  Writes
 * h = silu(x G^T) * (x U^T) (fp32) into the workspace.  sh_gate_w: [hidden]
 * act, the shared expert's sigmoid-gate row (mlp.shared_expert_gate.weight);
 * required when sh_w13 != NULL.  hidden % 512 == 0, inter % 128 == 0,
 * shared_inter % 128 == 0. */
int tm_moe_decode_gateup(const void *x, int64_t tokens, int hidden, int inter,
                         int n_experts, int top_k, int act_dtype, const uint8_t *w13,
                         const float *s13, const uint8_t *sh_w13, const float *sh_s13,
                         int shared_inter, const void *sh_gate_w, void *ws,
                         int64_t ws_bytes, void *stream);

/* K2 as tm_moe_decode_gateup; in addition each CTA, once its own weight
 * tile has landed, pulls its share of the packed down projections of the
 * same experts (w2 of the routed experts; sh_w2 when sh_w13 is set) from HBM
 * into L2, so that the tm_moe_decode_down_combine call that follows reads
 * them from L2.  Same arguments as tm_moe_decode_gateup plus w2 / sh_w2 (the
 * arrays later passed to tm_moe_decode_down_combine); same results bit for
 * bit. */
int tm_moe_decode_gateup_prefetch(const void *x, int64_t tokens, int hidden, int inter,
                                  int n_experts, int top_k, int act_dtype, const uint8_t *w13,
                                  const float *s13, const uint8_t *sh_w13, const float *sh_s13,
                                  int shared_inter, const void *sh_gate_w, const uint8_t *w2,
                                  const uint8_t *sh_w2, void *ws, int64_t ws_bytes, void *stream);

/* K3: down dequant-GEMV with the routing-weighted combine (+ the
 * sigmoid-gated shared expert, + an optional residual).  Replaces moe_seq's
 * down projection and weighted sum (execution/moe.py:18-19), the weighted
 * scatter-add of the multi-token path (moe.py:173-176) and the shared-expert
 * add (moe.py:79-85,196-202).  out[t] = residual[t] + sum_k topk_w[t,k] *
 * down_{idx[t,k]}(h) + gate_sh[t] * down_sh(h_sh).  residual may be NULL;
 * out: [tokens, hidden] act. */
int tm_moe_decode_down_combine(int64_t tokens, int hidden, int inter, int n_experts,
                               int top_k, int act_dtype, const void *topk_w,
                               const uint8_t *w2, const float *s2, const uint8_t *sh_w2,
                               const float *sh_s2, int shared_inter, const void *residual,
                               void *out, void *ws, int64_t ws_bytes, void *stream);

/* L2 prefetch of whole experts' packed weights: for each id in
 * expert_ids[0..n_ids) (device int64; ids outside [0, n_experts) are
 * skipped), bulk-prefetches bytes [id * expert_bytes, (id + 1) *
 * expert_bytes) of `weights` into L2.  A hint only: nothing is read into the
 * SMs or waited on, and no result depends on it.  Used to pull the experts a
 * later layer is predicted to route to (the w13 array of that layer,
 * expert_bytes = tm_packed_w13_bytes) into L2 while HBM would otherwise be
 * idle; no reference counterpart.  weights 16-byte aligned, expert_bytes a
 * multiple of 16. */
int tm_prefetch_experts_l2(const uint8_t *weights, int64_t expert_bytes, int n_experts,
                           const int64_t *expert_ids, int n_ids, void *stream);

/* ------------------------------------------------------------------------ */
/* K4: prefill (many tokens) as grouped GEMMs on the tcgen05 tensor cores.
 * Replaces the multi-token branch of MoEExecutor.execute_layer
 * (execution/moe.py:157-180): per active expert, h = silu(x G^T) * (x U^T),
 * y = h D^T, out[t] = residual[t] + sum_k topk_w[t,k] * y_{idx[t,k]}[t].
 * Weights are dequantised on chip to act dtype exactly as
 * ExpertLoader.dequantize_weight does (loader/expert_loader.py:150-160) and
 * multiplied with the activations on the tensor cores, fp32 accumulation;
 * h and y are rounded to act dtype (as the reference's F.linear outputs are).
 * Needs the routing plan of tm_router_topk / tm_route_plan in `ws`; uses the
 * workspace's h and partial-output regions.  act_dtype bf16 or fp16;
 * hidden % 256 == 0, inter % 128 == 0.  Optional shared expert (Qwen3.5;
 * moe.py:191-200): sh_w13/sh_s13/sh_w2/sh_s2 in the packed layout of one
 * expert, shared_inter == inter, gate row sh_gate_w [hidden] act; it runs as
 * one more group of the same GEMMs over every token and adds
 * sigmoid(x . sh_gate_w) * y_sh after the routed sum (all NULL / 0 = none;
 * needs n_experts > top_k).  |weight_scale_inv| must stay below 255 (the
 * on-chip dequantisation scales by 2^120 (bf16) / 2^8 (fp16)). */
int tm_moe_prefill_grouped(const void *x, int64_t tokens, int hidden, int inter, int n_experts,
                           int top_k, int act_dtype, const void *topk_w, const uint8_t *w13,
                           const float *s13, const uint8_t *w2, const float *s2,
                           const uint8_t *sh_w13, const float *sh_s13, const uint8_t *sh_w2,
                           const float *sh_s2, int shared_inter, const void *sh_gate_w,
                           const void *residual, void *out, void *ws, int64_t ws_bytes,
                           void *stream);

/* The same layer call as tm_moe_prefill_grouped (same arguments, plan,
 * workspace and results up to rounding) on FP8 tensor-core GEMMs
 * (tcgen05.mma kind::f8f6f4) that multiply the packed e4m3 weights as they
 * are stored: the tokens enter as two e4m3 terms (exact for bf16), each
 * 128 x 128 weight block's scale is applied to its fp32 partial sum, g, u,
 * silu(g) and h are rounded to bf16 as the reference rounds them
 * (execution/moe.py:157-202).  Built for few tokens per expert (expert-parallel
 * owners, batched decode); bf16 activations only; hidden and inter multiples
 * of 128. */
int tm_moe_grouped_f8(const void *x, int64_t tokens, int hidden, int inter, int n_experts, int top_k,
                      int act_dtype, const void *topk_w, const uint8_t *w13, const float *s13,
                      const uint8_t *w2, const float *s2, const uint8_t *sh_w13, const float *sh_s13,
                      const uint8_t *sh_w2, const float *sh_s2, int shared_inter, const void *sh_gate_w,
                      const void *residual, void *out, void *ws, int64_t ws_bytes, void *stream);

/* Weighted combine of per-slot expert outputs in top-k order:
 * out[t] = residual[t] + sum_r topk_w[t,r] * y[pair_slot[t*top_k + r]]
 * (fp32 sums, slots < 0 skipped).  Replaces the weighted scatter-add of
 * execution/moe.py:173-176 where the expert outputs were computed elsewhere
 * (the expert-parallel path: rows come back from the ranks owning the
 * experts).  y: [P][hidden] act; pair_slot: int32 [tokens*top_k]; bf16/fp16;
 * hidden % 8 == 0. */
int tm_combine_slots(const void *y, const void *topk_w, const int32_t *pair_slot, int64_t tokens,
                     int hidden, int top_k, int act_dtype, const void *residual, void *out,
                     void *stream);

/* ------------------------------------------------------------------------ */
/* One whole decode layer without a caller workspace.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory for a
 * workspace (a C/FFI host without a device allocator, or a serving process
 * whose memory pool already owns the free HBM; cudaMalloc would also
 * synchronise the device).  Runs tm_router_topk, tm_moe_decode_gateup and
 * tm_moe_decode_down_combine (same arguments and results as those) on a
 * library-owned static device array of TM_NOALLOC_SCRATCH_BYTES per GPU, held
 * by every GPU that loads the library until exit, and allocates nothing.
 *   - Calls whose tm_workspace_bytes(tokens, n_experts, top_k, hidden, inter,
 *     shared_inter) exceeds TM_NOALLOC_SCRATCH_BYTES are rejected with
 *     TM_ERR_WORKSPACE.  8 MiB covers 64 tokens of a Qwen3-30B-A3B layer
 *     (E 128, top-8, H 2048, I 768: 6.1 MiB) and of a Qwen3.5 layer (E 256,
 *     top-8, H 2048, I 512, shared I 512: 5.9 MiB); larger shapes fit fewer
 *     tokens (E 512, top-10, H 4096, I 1024 needs 14.2 MiB at 64 tokens), so
 *     check your own shape with tm_workspace_bytes.
 *   - It always runs the decode kernels (K1, K2 with the L2 prefetch of the
 *     down projections, K3), never the tcgen05 grouped GEMMs that the
 *     workspace path switches to from 16 tokens: calls of 16-64 tokens are
 *     slower here than through the workspace entry points.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current) and caches it with the
 *     device's current CUDA context; a call under another context looks it up
 *     again.  Make that first call before any stream capture.
 *   - Every call shares the array; each call clears its header first.  Calls
 *     that overlap on the GPU (other streams or threads on the same device)
 *     race on it: order them on one stream.
 *   - status: optional device uint32, receives the TM_STATUS_* bits of this
 *     call (NULL to skip).  sh_w13 and sh_w2 are both set or both NULL. */
#define TM_NOALLOC_SCRATCH_BYTES (8ll << 20)
int tm_moe_decode_layer_noalloc(const void *x, int64_t tokens, int hidden, int inter,
                                int n_experts, int top_k, int act_dtype, const void *router_w,
                                const uint8_t *w13, const float *s13, const uint8_t *w2,
                                const float *s2, const uint8_t *sh_w13, const float *sh_s13,
                                const uint8_t *sh_w2, const float *sh_s2, int shared_inter,
                                const void *sh_gate_w, const void *residual, int64_t *topk_idx,
                                void *topk_w, void *out, uint32_t *status, void *stream);

/* ------------------------------------------------------------------------ */
/* Dense FP8 block-scaled linear (attention q/k/v/o and other projections of
 * an FP8 checkpoint).  Replaces ExpertLoader.load_weight's dequantisation
 * (loader/expert_loader.py:109-112, arithmetic of :150-160) followed by
 * F.linear for the projections of execution/layouts/qwen3.py:6-17:
 *   out[t, n] = sum_k x[t, k] * W[n, k] * scale_inv[n/128, k/128]
 *               (+ residual[t, n]), fp32 accumulation, rounded once to act.
 * W is e4m3 [out_features, in_features] packed by tm_pack_linear
 * (tm_packed_w2_bytes(out_features, in_features) bytes, the layout of one
 * expert's down projection); scale_inv is the checkpoint's fp32
 * [out_features/128, in_features/128] as is.  x [tokens, in_features] and out
 * [tokens, out_features] act (bf16 or fp16 on the tensor-core kernel; fp32 on a
 * CUDA-core kernel that dequantises each weight as the reference's fp32
 * load_weight does); in_features % 512 == 0 (at most
 * 6144), out_features % 128 == 0.  One pass over W per call (decode-sized
 * calls are HBM-bound).  status: optional device uint32 for TM_STATUS_*. */
int tm_pack_linear(const uint8_t *w, int out_features, int in_features, uint8_t *w_packed, void *stream);
int tm_fp8_linear(const void *x, int64_t tokens, int in_features, int out_features, int act_dtype,
                  const uint8_t *w_packed, const float *scale_inv, const void *residual, void *out,
                  uint32_t *status, void *stream);
/* One token, bf16/fp16: RMSNorm of x (tm_rmsnorm's arithmetic, the same bits)
 * then tm_fp8_linear of the normalised row, in one kernel (hidden 2048 or
 * 4096): the decode step's input norm fused into the q/k/v projection. */
int tm_rmsnorm_fp8_linear(const void *x, int hidden, int act_dtype, const void *norm_w, float eps,
                          int out_features, const uint8_t *w_packed, const float *scale_inv,
                          const void *residual, void *out, uint32_t *status, void *stream);

/* ------------------------------------------------------------------------ */
/* The rest of a Qwen3-MoE decode step (the full-model loop around the MoE
 * path: runtime/engine.py:98-162, execution/layer_executor.py:137-170, over
 * the Hugging Face Qwen3-MoE modules).  Every call reads its inputs from
 * device memory (token ids and positions included), so a whole decode step
 * can be captured in one CUDA graph and replayed with no host round trip.
 * head_dim is 128.  Workspaces are caller-owned, zeroed once (their
 * counters reset themselves) and must not be shared by overlapping calls. */

/* out[t] = embed_tokens[ids[t]] (bf16 table [vocab][hidden] -> act).  An id
 * outside [0, vocab) writes zeros and sets TM_STATUS_BAD_TOKEN_ID in *status
 * (optional). */
int tm_embed(const int64_t *ids, int64_t tokens, const void *table_bf16, int hidden, int64_t vocab,
             int act_dtype, void *out, uint32_t *status, void *stream);
/* RMSNorm of each token row (Qwen3MoeRMSNorm): fp32 mean of squares,
 * round(x * rsqrt(mean + eps)) to act, times weight (act), rounded. */
int tm_rmsnorm(const void *x, int64_t tokens, int hidden, int act_dtype, const void *weight, float eps,
               void *out, void *stream);
/* qkv [tokens][(n_heads + 2 n_kv_heads) * 128] (fused q/k/v projection output):
 * q heads get RMSNorm (q_norm_w) and the rotary embedding at positions[t] ->
 * q_out [tokens][n_heads][128]; k heads RMSNorm (k_norm_w) + rotary ->
 * k_cache[kv][positions[t]]; v heads -> v_cache[kv][positions[t]].  Caches of
 * one layer are [n_kv_heads][max_len][128] act; rope_table [max_len][2][128]
 * act holds cos then sin per position (Qwen3MoeRotaryEmbedding's values).
 * A position outside [0, max_len) skips the token and sets
 * TM_STATUS_BAD_TOKEN_ID. */
int tm_qk_rope_kv(const void *qkv, int64_t tokens, int n_heads, int n_kv_heads, int head_dim, int act_dtype,
                  const void *q_norm_w, const void *k_norm_w, float eps, const void *rope_table,
                  const int64_t *positions, int64_t max_len, void *q_out, void *k_cache, void *v_cache,
                  uint32_t *status, void *stream);
/* One query token's attention over cache positions [0, *position] (GQA, query
 * head h reads KV head h / (n_heads / n_kv_heads)): softmax(scale q.k) v in
 * fp32, out [n_heads * 128] act.  The positions are split over `splits` CTAs
 * per KV head and merged by the last one. */
int64_t tm_attn_decode_workspace_bytes(int n_heads, int n_kv_heads, int splits);
int tm_attn_decode(const void *q, const void *k_cache, const void *v_cache, const int64_t *position,
                   int64_t max_len, int n_heads, int n_kv_heads, int head_dim, int act_dtype, float scale,
                   int splits, void *out, void *ws, int64_t ws_bytes, void *stream);
/* One query token, bf16/fp16: tm_qk_rope_kv and tm_attn_decode in one launch.
 * qkv is the fused q/k/v projection output [(n_heads + 2 n_kv_heads) * 128];
 * the query heads get q_norm + rotary inside the attention kernel, this
 * step's k (k_norm + rotary) and v are appended to k_cache / v_cache at
 * *position and attended to; same bits as the two calls.  A position at or
 * past max_len appends nothing (the separate call flags it). */
int tm_qk_rope_attn_decode(const void *qkv, const void *q_norm_w, const void *k_norm_w, float eps,
                           const void *rope_table, const int64_t *position, int64_t max_len, int n_heads,
                           int n_kv_heads, int head_dim, int act_dtype, float scale, int splits, void *k_cache,
                           void *v_cache, void *out, void *stream);
/* Batched decode (one query token per sequence, bf16/fp16): sequence b reads
 * q + b * n_heads * 128 and writes out + b * n_heads * 128, its caches start
 * at k_cache / v_cache + b * kv_batch_stride elements (each
 * [n_kv_heads][max_len][128], as tm_qk_rope_kv writes them) and its context is
 * positions[b] + 1 (ragged over the batch).  `splits` (<= 16 used) CTAs per
 * (sequence, KV head) form one thread-block cluster and merge through
 * distributed shared memory; no workspace.  The reference's KVCache
 * (cache/kv_cache.py:28-54) appends [batch, kv_heads, new, 128] slices with
 * one sequence length for the whole batch and attends through Hugging Face
 * attention; here every sequence has its own length (the expert-parallel
 * batched-decode configuration). */
int tm_attn_decode_batched(const void *q, const void *k_cache, const void *v_cache, const int64_t *positions,
                           int batch, int64_t kv_batch_stride, int64_t max_len, int n_heads, int n_kv_heads,
                           int head_dim, int act_dtype, float scale, int splits, void *out, void *stream);
/* LM head and greedy choice: logits = x . W^T (W bf16 [vocab][hidden], fp32
 * accumulation, rounded to act for 16-bit act), optional logits output (act
 * [vocab], NULL to skip), *token = index of the largest logit (lowest index
 * among equal maxima, as torch.argmax). */
int64_t tm_lm_head_workspace_bytes(void);
int tm_lm_head_argmax(const void *x, int hidden, int act_dtype, const void *w_bf16, int64_t vocab, void *logits,
                      int64_t *token, void *ws, int64_t ws_bytes, void *stream);

/* ------------------------------------------------------------------------ */
/* Qwen3.5 linear attention, one decode token per sequence (batch rows).
 * Replaces, for a "linear_attention" layer with a cached state, the core of
 * Qwen3_5MoeGatedDeltaNet.forward that execution/layer_executor.py:134-139
 * calls with the reference's Qwen35Cache (cache/qwen35_cache.py:43-64):
 * torch_causal_conv1d_update, the gates beta = sigmoid(b) and
 * g = -exp(A_log) * softplus(a + dt_bias), torch_recurrent_gated_delta_rule
 * with q/k l2-normalised in the act dtype and q scaled by 1/sqrt(128), and
 * Qwen3_5MoeRMSNormGated (transformers 5.5.0 modeling_qwen3_5_moe.py:176-191,
 * :211-226, :315-354, :484-533).  The in_proj_* and out_proj GEMMs stay with
 * the caller.
 *   qkv [batch][2*n_k_heads*128 + n_v_heads*128] (q heads, k heads, v heads);
 *   z [batch][n_v_heads*128]; a, b [batch][n_v_heads]; conv_w
 *   [conv_dim][conv_kernel] (conv1d.weight without its middle axis); norm_w
 *   [128]; all act dtype.  A_log, dt_bias: fp32 [n_v_heads].
 *   conv_state_in -> conv_state_out: [batch][conv_dim][conv_kernel] act, the
 *   state shifted left with this token appended; the two must not overlap
 *   (value heads that share a key head read the old q/k columns while one of
 *   them writes the new ones): keep two buffers and swap them per step.
 *   recurrent_state: fp32 [batch][n_v_heads][128][128] (S[d_k][d_v]), updated
 *   in place, 16-byte aligned.
 *   out: [batch][n_v_heads*128] act, the gated-normed output (out_proj input).
 * head_k_dim = head_v_dim = 128, n_v_heads a multiple of n_k_heads,
 * conv_kernel 1..8, batch <= 65535. */
int tm_gdn_decode(const void *qkv, const void *z, const void *a, const void *b, int64_t batch, int n_k_heads,
                  int n_v_heads, int head_k_dim, int head_v_dim, int conv_kernel, int act_dtype,
                  const void *conv_w, const float *A_log, const float *dt_bias, const void *norm_w, float eps,
                  const void *conv_state_in, void *conv_state_out, float *recurrent_state, void *out,
                  void *stream);

/* ------------------------------------------------------------------------ */
/* Expert parallelism over NVLink peer memory (no counterpart in the reference,
 * which runs batch 1 on one device: runtime/engine.py:103-107,158; per token
 * the arithmetic is MoEExecutor.execute_layer, execution/moe.py:99-208).
 * The experts of a layer are sharded over `world` ranks of one node (one
 * process per GPU; rank r owns experts [r*E/world, (r+1)*E/world)).  Every
 * rank creates a context (one device buffer of identical layout), exchanges
 * the 64-byte IPC handles with its peers by any host means and connects.
 * One layer call on every rank, in this order on one stream:
 *   tm_router_topk(x, ..., ws)            top-k + routing plan of the local tokens
 *   tm_ep_dispatch(ctx, x, T, idx, ws)    rows -> the owners' buffers (peer stores)
 *   tm_ep_experts(ctx, local experts, owner_ws)
 *                                         wait for all sources, grouped GEMMs on
 *                                         the received rows, outputs -> sources
 *   tm_ep_combine(ctx, w, T, ws, residual, out)
 *                                         wait for all owners, weighted sum
 * No host synchronisation: the sequence is CUDA-graph capturable.  Every
 * device-side wait is bounded (tm_ep_set_timeout, default 2 s); on expiry
 * TM_STATUS_TIMEOUT is set in the context status (tm_ep_status) and the call's
 * outputs are invalid.  An owner that timed out waiting for a source returns
 * nothing and tells every source, which sets TM_STATUS_PEER_FAILED: each rank
 * whose outputs of the call are invalid sees a status bit.  A context whose
 * status showed either bit may still receive late rows of the failed call:
 * disconnect and destroy it on every rank (host barriers around both) and
 * create a new one before the next call.  Tokens per call may differ between
 * ranks (each at most max_tokens).  bf16/fp16 activations; hidden % 256 == 0,
 * inter % 128 == 0. */
#define TM_EP_MAX_RANKS 8
#define TM_EP_HANDLE_BYTES 64
typedef struct tm_ep_ctx tm_ep_ctx;
/* Bytes of the device buffer each rank allocates (for reporting). */
int64_t tm_ep_buffer_bytes(int world, int64_t max_tokens, int n_experts, int top_k, int hidden, int act_dtype);
/* Allocate and zero this rank's buffer on the current device; writes its IPC
 * handle (TM_EP_HANDLE_BYTES, host memory) to handle_out. */
int tm_ep_create(int rank, int world, int n_experts, int top_k, int hidden, int inter, int act_dtype,
                 int64_t max_tokens, void *handle_out, tm_ep_ctx **out);
/* Map the peers' buffers: handles = world x TM_EP_HANDLE_BYTES in rank order
 * (host memory; this rank's own entry is ignored). */
int tm_ep_connect(tm_ep_ctx *ctx, const void *handles);
/* Alternative to tm_ep_connect for hosts that map peer memory themselves:
 * peer_bases[r] = rank r's buffer in this process (own entry ignored). */
int tm_ep_connect_ptrs(tm_ep_ctx *ctx, void *const *peer_bases);
/* This rank's buffer (device pointer), for tm_ep_connect_ptrs of other contexts. */
void *tm_ep_local_buffer(tm_ep_ctx *ctx);
int tm_ep_set_timeout(tm_ep_ctx *ctx, int64_t timeout_ns);
/* Synchronises the device and unmaps the peers' buffers.  Call it on every
 * rank after a host barrier (no peer may still be in a layer call). */
int tm_ep_disconnect(tm_ep_ctx *ctx);
/* Frees this rank's buffer and the context (disconnecting first if needed).
 * Call it after every rank has disconnected (a second host barrier). */
int tm_ep_destroy(tm_ep_ctx *ctx);
/* Workspace bytes tm_ep_experts needs (zero it once with tm_workspace_init). */
int64_t tm_ep_owner_workspace_bytes(const tm_ep_ctx *ctx);
/* Copy the context's status word (TM_STATUS_* bits) to *host_status and clear
 * it; synchronises `stream`. */
int tm_ep_status(tm_ep_ctx *ctx, uint32_t *host_status, void *stream);
/* Source: after tm_router_topk on `ws` for these `tokens`, send every routed
 * (token, expert) row to the expert's owner.  topk_idx: the router's output. */
int tm_ep_dispatch(tm_ep_ctx *ctx, const void *x, int64_t tokens, const int64_t *topk_idx, void *ws,
                   int64_t ws_bytes, void *stream);
/* Owner: wait for every source's rows, run this rank's experts on them (packed
 * layout of tm_pack_experts for the n_experts/world local experts) and return
 * each output row to its source. */
int tm_ep_experts(tm_ep_ctx *ctx, const uint8_t *w13, const float *s13, const uint8_t *w2, const float *s2,
                  void *owner_ws, int64_t owner_ws_bytes, void *stream);
/* Source: wait for every owner's outputs, then out = residual + sum_k w * y in
 * top-k order (residual may be NULL). */
int tm_ep_combine(tm_ep_ctx *ctx, const void *topk_w, int64_t tokens, void *ws, int64_t ws_bytes,
                  const void *residual, void *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* TURBOMOE_H */
