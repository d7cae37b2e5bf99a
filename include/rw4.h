/*
 * rw4.h -- C ABI of the RW4 4-bit hot path for B200 (sm_100a).
 *
 * RW4 is RocketLLM's int4 codec applied to Linear weights: a weight W[N, K] is grouped along K in
 * groups of 64, each group stored as 4-bit codes (two per byte, even index in the low nibble),
 * an fp16 scale and an fp16 zero; the value is code * scale + zero computed in fp32
 * (rocketllm/quant/kv_cache.py:190-272).  Device layout is the checkpoint layout, row-major:
 *   packed  uint8   [N, K/2]
 *   scale   fp16    [N, K/64]
 *   zero    fp16    [N, K/64]
 *
 * Conventions for every entry point:
 *   - plain pointers and sizes, no framework types; bf16/fp16 buffers are passed as void*;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream); every launch
 *     goes on that stream and no call synchronises the device unless it says so;
 *   - the return value is a status: 0 (RW4_OK) or a negative RW4_E* code; a human-readable
 *     message for the last failure on the calling thread is available from rw4_last_error();
 *   - shape and alignment violations are rejected before any launch (RW4_EINVAL);
 *   - the library never frees caller memory; caller buffers must stay live until the work
 *     queued on `stream` has completed.
 */
#ifndef RW4_H
#define RW4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define RW4_OK 0
#define RW4_EINVAL (-1)      /* bad shape, pointer, alignment or argument */
#define RW4_ECUDA (-2)       /* a CUDA runtime call failed; see rw4_last_error() */
#define RW4_ENOMEM (-3)      /* host or device allocation failed */
#define RW4_ETIMEOUT (-4)    /* a bounded wait gave up */
#define RW4_EBUSY (-5)       /* no free slot / resource in use */
#define RW4_EUNSUPPORTED (-6)

/* element types for out_dtype / w_dtype arguments */
#define RW4_F32 0
#define RW4_BF16 1
#define RW4_F16 2

/* ABI version (major * 100 + minor). */
int rw4_version(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated to n). Returns the
 * full message length. */
int rw4_last_error(char* buf, size_t n);

/*
 * rw4_dequant: expand a packed weight to out[N, K] (row-major, dtype out_dtype).
 * Bit-exact with QuantizedTensor.dequantize() (rocketllm/quant/kv_cache.py:249-257): fp32
 * code*scale+zero, narrowed to K columns, then cast with round-to-nearest-even.
 * `packed` has ceil(K/group)*group/2 bytes per row (a ragged K keeps the reference's padding).
 * Replaces the reference's dequant-to-scratch seam QuantBackend.prepare_layer
 * (rocketllm/quant/registry.py:529-535; rocketllm/base.py:848-855).
 */
int rw4_dequant(const uint8_t* packed, const void* scale_f16, const void* zero_f16, int64_t N,
                int64_t K, int32_t group, void* out, int32_t out_dtype, void* stream);

/*
 * rw4_quantize: encode w[N, K] (dtype w_dtype: RW4_F32, RW4_BF16 or RW4_F16) into
 * packed/scale/zero, bit-exact with quantize(w, axis=1, group_size=group)
 * (rocketllm/quant/kv_cache.py:190-221), including the scale arithmetic in the input dtype and
 * the repeat-last-value padding of a ragged K.
 * Output rows have ceil(K/group) groups.
 */
int rw4_quantize(const void* w, int32_t w_dtype, int64_t N, int64_t K, int32_t group,
                 uint8_t* packed, void* scale_f16, void* zero_f16, void* stream);

/*
 * rw4_linear: y[M, N] = x[M, K] . W[N, K]^T, bf16 in and out, fp32 accumulation, W in RW4.
 * Replaces the nn.Linear / F.linear call a transformers module makes on a dequantized weight
 * (transformers models/llama/modeling_llama.py:171-184 via rocketllm/base.py:848-855).
 * M <= 16 runs the dequant-GEMV; 17-64 rows the GEMV in 16-row batch slices, or for 49-64 rows
 * the tcgen05 decode GEMM where the weight has enough 128-row tiles; larger M the tcgen05 GEMM
 * (rw4_linear_path).  The GEMV and the decode GEMM multiply by the exact fp32 weight
 * code * scale + zero; the GEMV gives each row of y the same bits at every M <= 16, the decode GEMM
 * at every M of one column tile (17-32, 33-64) -- a row's output does not depend on the rows beside
 * it; the GEMM multiplies by the reference's bf16-rounded weight (dequantize().to(bfloat16),
 * rocketllm/quant/kv_cache.py:257).  group must be 64 and K a multiple of 64; x, y and packed
 * must be 16-byte aligned, scale and zero 8-byte aligned.  Most GEMV calls need a workspace
 * (rw4_linear_workspace_size); this entry point takes it from the device's stream-ordered memory
 * pool on `stream` and returns it there (rw4_linear_ws takes a caller-owned one instead).
 */
int rw4_linear(const void* x_bf16, int64_t M, int64_t K, const uint8_t* packed,
               const void* scale_f16, const void* zero_f16, int64_t N, int32_t group,
               void* y_bf16, void* stream);

/* Which kernel rw4_linear would launch for (M, K, N): 1 = GEMV, 2 = tcgen05 GEMM,
 * 3 = GEMV over 16-row slices, 4 = tcgen05 decode GEMM (picked for 49-64 rows; runs 17-64 rows
 * with K % 512 == 0 and N >= 12288). Negative on invalid shapes. Host-only, launches nothing. */
int rw4_linear_path(int64_t M, int64_t K, int64_t N);

/* rw4_linear on a given path (1 or 3: GEMV / GEMV slices, 2: tcgen05 GEMM, which needs M > 16,
 * 4: tcgen05 decode GEMM, which needs the shapes above)
 * instead of the one rw4_linear_path picks; for tests and measurements of each kernel. */
int rw4_linear_on_path(const void* x_bf16, int64_t M, int64_t K, const uint8_t* packed,
                       const void* scale_f16, const void* zero_f16, int64_t N, int32_t group,
                       void* y_bf16, int32_t path, void* stream);

/* Bytes of device workspace rw4_linear_ws needs for (M, K, N) on `path` (0 = the path
 * rw4_linear_path picks): the converted activations of the GEMV and the decode GEMM (about
 * 2*M*K bytes; 0 for one row that the GEMV converts itself, and for the GEMM).  Host-only.  No
 * reference counterpart: the
 * reference's F.linear takes no workspace. */
int rw4_linear_workspace_size(int64_t M, int64_t K, int64_t N, int32_t path, size_t* bytes);

/* rw4_linear with a caller-owned device workspace of workspace_bytes (>= the size above, 256-byte
 * aligned; may be NULL when that size is 0) on `path` (0 = rw4_linear_path's choice).  The
 * workspace is written and read by the work queued on `stream`; it must not be shared with work
 * that can run at the same time.  Same replacement as rw4_linear. */
int rw4_linear_ws(const void* x_bf16, int64_t M, int64_t K, const uint8_t* packed,
                  const void* scale_f16, const void* zero_f16, int64_t N, int32_t group,
                  void* y_bf16, int32_t path, void* workspace, size_t workspace_bytes,
                  void* stream);

/* ---------------------------------------------------------------------------------------------
 * Decode-step kernels around the projections of a Llama-family decoder layer, each replacing a
 * chain of small transformers ops with one launch and the same bf16 rounding sequence
 * (transformers models/llama/modeling_llama.py).  All bf16 unless stated.
 *
 * rw4_rmsnorm: y[r] = weight * bf16(x[r] * rsqrt(mean(x[r]^2) + eps)) (LlamaRMSNorm, :48-68);
 *   rows <= 65535.
 * rw4_rope_kv: rotary embedding of the q and k heads of `rows` token rows (one per sequence) with
 *   bf16 cos / sin [rows, head_dim] (apply_rotary_pos_emb, :78-112), q written to q_out
 *   [rows, heads, head_dim], k and v written into the static caches [rows, kv_heads, cache_len,
 *   head_dim] at position *pos (DEVICE int64: a CUDA graph can replay it); q, k, v are row-major
 *   with row stride ld elements (the slices of one concatenated q|k|v projection).  Replaces
 *   apply_rotary_pos_emb + StaticCache.update's index_copy_.
 * rw4_silu_mul: out[r, i] = bf16(bf16(silu(g)) * u), g = gate_up[r, i], u = gate_up[r, I + i]
 *   (act_fn(gate_proj(x)) * up_proj(x) of a concatenated gate|up projection, :171-184).
 * rw4_linear_residual_ws: y = bf16(residual + bf16(x . W^T)) for M <= 64 (the kernel rw4_linear
 *   would run -- the GEMV, or the decode GEMM -- with the decoder layer's residual add in its
 *   epilogue); residual [M, N] may be y itself (in place) when K is a multiple of 512.
 *   Workspace as rw4_linear_ws.
 * ------------------------------------------------------------------------------------------- */
int rw4_rmsnorm(const void* x, const void* weight, int64_t rows, int64_t H, float eps, void* y,
                void* stream);
int rw4_rope_kv(const void* q, const void* k, const void* v, int64_t ld, int32_t rows,
                int32_t heads, int32_t kv_heads, int32_t head_dim, const void* cos_bf16,
                const void* sin_bf16, const int64_t* pos, int64_t cache_len, void* q_out,
                void* k_cache, void* v_cache, void* stream);
int rw4_silu_mul(const void* gate_up, int64_t rows, int64_t I, void* out, void* stream);
/* rw4_linear_rmsnorm_ws: y = x_n . W^T with x_n = rw4_rmsnorm(x, norm_weight, eps) for M <= 64
 *   (a decoder layer's input_layernorm / post_attention_layernorm followed by its first
 *   projection); with K % 512 == 0 the norm runs inside the activation conversion (the one-row
 *   GEMV's prologue, or the x-prep pass of more rows: no separate launch, the same bits as the
 *   two calls), otherwise rw4_rmsnorm first.
 *   norm_weight bf16 [K], 16-byte aligned; workspace of rw4_linear_rmsnorm_workspace_size bytes,
 *   256-byte aligned. */
int rw4_linear_rmsnorm_workspace_size(int64_t M, int64_t K, int64_t N, size_t* bytes);
int rw4_linear_rmsnorm_ws(const void* x_bf16, int64_t M, int64_t K, const void* norm_weight,
                          float eps, const uint8_t* packed, const void* scale_f16,
                          const void* zero_f16, int64_t N, int32_t group, void* y_bf16,
                          void* workspace, size_t workspace_bytes, void* stream);
/* rw4_linear_rmsnorm_swiglu_ws: y[M, N/2] = act_fn(x_n . W_gate^T) * (x_n . W_up^T), x_n as in
 *   rw4_linear_rmsnorm_ws, for a [gate; up] weight of N rows (gate rows first): a Llama MLP's
 *   post_attention_layernorm, gate_proj, up_proj and act_fn(gate) * up (LlamaMLP.forward,
 *   transformers models/llama/modeling_llama.py), the bits of rw4_linear_rmsnorm_ws followed by
 *   rw4_silu_mul.  One launch where the GEMV's launch shape for the weight has no K split and the
 *   call takes the GEMV (K % 512 == 0; M <= 48, or no decode-GEMM shape); otherwise those two
 *   calls through the workspace (rw4_linear_rmsnorm_swiglu_workspace_size bytes, 256-byte
 *   aligned). */
int rw4_linear_rmsnorm_swiglu_workspace_size(int64_t M, int64_t K, int64_t N, size_t* bytes);
int rw4_linear_rmsnorm_swiglu_ws(const void* x_bf16, int64_t M, int64_t K,
                                 const void* norm_weight, float eps, const uint8_t* packed,
                                 const void* scale_f16, const void* zero_f16, int64_t N,
                                 int32_t group, void* y_bf16, void* workspace,
                                 size_t workspace_bytes, void* stream);
/* rw4_decode_attention: one decode step's attention over a bf16 static KV cache.  q [batch,
 *   heads, head_dim] (the step's rotated queries), k_cache / v_cache [batch, kv_heads, cache_cap,
 *   head_dim] (StaticCache layout, the step's own key and value already written at *pos), out
 *   [batch, heads, head_dim] = softmax(scaling q K^T) V over positions 0 .. *pos of each sequence,
 *   grouped-query heads (heads / kv_heads <= 8), head_dim 64 or 128, all bf16 and 16-byte aligned.
 *   *pos is read on the device (int64), so a captured graph replays the call unchanged as the
 *   position advances.  Stands for transformers' sdpa_attention_forward over a StaticCache with
 *   the causal mask of a one-token step (models/llama/modeling_llama.py), within bf16 rounding. */
int rw4_decode_attention(const void* q, int32_t batch, int32_t heads, int32_t kv_heads,
                         int32_t head_dim, const void* k_cache, const void* v_cache,
                         int64_t cache_cap, const int64_t* pos, float scaling, void* out,
                         void* stream);
int rw4_linear_residual_ws(const void* x_bf16, int64_t M, int64_t K, const uint8_t* packed,
                           const void* scale_f16, const void* zero_f16, int64_t N, int32_t group,
                           const void* residual, void* y_bf16, void* workspace,
                           size_t workspace_bytes, void* stream);
/* rw4_argmax_rows: the greedy token choice of a decode step, out[r] (int64) = the index of the
 *   largest of row r's V bf16 scores (row stride ld elements), the first index among equal maxima,
 *   a NaN counting as larger than every number -- torch.argmax(scores, dim=-1), which the
 *   reference's generate() reaches through the model's own greedy search (rocketllm/base.py:
 *   2014-2044 -> transformers generation/utils.py, the greedy branch of _sample).  rows <= 65535,
 *   V <= 2^31 - 2049.  One launch, one cluster of CTAs per row, no scratch. */
int rw4_argmax_rows(const void* scores_bf16, int64_t rows, int64_t V, int64_t ld, int64_t* out,
                    void* stream);

/* rw4_linear_noalloc: rw4_linear for M <= 64 (the GEMV) that allocates nothing.  No counterpart in
 * the reference.  For callers that cannot allocate device memory per call: a host that plans every
 * byte of VRAM up front (a streaming engine sizing its layer slots from measured free memory, a
 * serving process with a fixed memory plan) or a C caller with no allocator to hand a workspace
 * from.  The scratch the GEMV needs for its converted activations is a fixed 4 MiB array in the
 * library's device image, reserved on every GPU that loads the library until the process exits;
 * a call needing more (about M*K > 2M values) or M > 64 is rejected with RW4_EINVAL.  The first
 * call on a device looks up that array's device address (cudaGetSymbolAddress), so make it before
 * any stream capture.  All calls share the array: calls whose work can overlap on the GPU race and
 * must be serialised by the caller.  The array keeps the last call's contents; nothing has to be
 * cleared between calls.  Same arithmetic and bits as rw4_linear for the same M. */
int rw4_linear_noalloc(const void* x_bf16, int64_t M, int64_t K, const uint8_t* packed,
                       const void* scale_f16, const void* zero_f16, int64_t N, int32_t group,
                       void* y_bf16, void* stream);

/* Reads the library's device status word on the current device after the work queued on `stream`
 * (synchronises that stream): bit 1 = a bounded wait inside a kernel gave up (the kernel returned
 * early and its outputs are invalid), bit 2 = a tensor-memory allocation failed.  clear != 0 resets
 * the word.  No reference counterpart: the reference has no device kernels that can wait. */
int rw4_device_status(uint32_t* word, int32_t clear, void* stream);

/* Diagnostic (no reference counterpart): one block runs the library's bounded mbarrier wait on a
 * barrier that completes (arrive != 0) or that nothing completes (arrive == 0).  In the second case
 * the wait gives up after its limit (1 s), sets bit 1 of the device status word and the kernel
 * returns -- how every kernel here reports a copy that never landed, without trapping or hanging. */
int rw4_wait_selftest(int32_t arrive, void* stream);

/* ---------------------------------------------------------------------------------------------
 * MoE routed experts.  Together these replace the experts forward the reference streams
 * (transformers models/mixtral/modeling_mixtral.py:62-98, reached through rocketllm/base.py's
 * expert hooks :1083-1464): permute -> gather -> grouped RW4 GEMV (gate/up with SwiGLU) -> grouped
 * RW4 GEMV (down) -> combine.  Routing indices come from the model's own router unchanged.
 * ------------------------------------------------------------------------------------------- */

/*
 * rw4_moe_permute: stable counting sort of the T*k (token, slot) pairs by expert id.
 * topk_idx int64 [T, k].  Writes perm int32 [T*k] (perm[row] = t*k + j; rows of expert e are
 * offsets[e] .. offsets[e+1]-1, in increasing t*k+j order), inv int32 [T*k] (inv[t*k+j] = row;
 * may be NULL) and offsets int32 [E+1].  Ids outside [0, E) are dropped: their inv entry is -1,
 * offsets[E] counts only valid slots and the unused tail of perm is -1.  E <= 4096.
 */
int rw4_moe_permute(const int64_t* topk_idx, int64_t T, int32_t k, int32_t E, int32_t* perm,
                    int32_t* inv, int32_t* offsets, void* stream);

/* rw4_moe_gather: x_perm[row] = x[perm[row] / k] (zeros where perm[row] < 0), bf16 rows of H
 * values, H % 8 == 0. */
int rw4_moe_gather(const void* x_bf16, const int32_t* perm, int64_t T, int32_t k, int64_t H,
                   void* x_perm_bf16, void* stream);

/*
 * rw4_moe_grouped: for every expert e, y_perm[rows of e] = act(x_perm[rows of e] . W_e^T); an
 * expert with no routed rows is never read.  Weights are per-expert RW4 tensors W_e [N, K]; their
 * device pointers are passed in HOST arrays packed_e[E], scale_e[E], zero_e[E] (the host encodes
 * one TMA descriptor per expert).  `offsets` is the DEVICE int32 [E+1] from rw4_moe_permute;
 * max_rows bounds any expert's row count (T*k is always safe).  group 64, K % 512 == 0.
 * act = 0: y_perm [T*k, N].
 * act = 1: stacked gate/up weight, N = 2*I: y_perm [T*k, I] = bf16(silu(bf16(g)) * bf16(u)) with
 *          g = x.W[i], u = x.W[I+i] (the rounding sequence of the bf16 model's act_fn(gate) * up).
 */
int rw4_moe_grouped(const void* x_perm_bf16, const int32_t* offsets, int32_t E, int64_t max_rows,
                    const uint8_t* const* packed_e, const void* const* scale_e,
                    const void* const* zero_e, int64_t K, int64_t N, int32_t group, int32_t act,
                    void* y_perm_bf16, void* stream);

/*
 * rw4_moe_combine: out[t] = sum over the token's k slots of w[t, j] * y_perm[inv[t*k+j]], visiting
 * slots in ascending expert id (topk_idx; NULL = slot order) and rounding to bf16 after every
 * product and add -- the order and rounding of the reference's index_add_ into a bf16 tensor.
 * No atomics; deterministic.  topk_w fp32 (w_dtype RW4_F32) or bf16 [T, k]; k <= 8; H % 8 == 0.
 */
int rw4_moe_combine(const void* y_perm_bf16, const int32_t* inv, const int64_t* topk_idx,
                    const void* topk_w, int32_t w_dtype, int64_t T, int32_t k, int64_t H,
                    void* out_bf16, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Device-side routing into the expert cache.  Together these replace the routed-set read-back
 * and host-issued expert reads of the reference's streaming MoE path (rocketllm/moe/router.py:
 * 88-93, rocketllm/base.py:1375-1464, rocketllm/moe/expert_cache.py:261-316): nothing on the host
 * waits for the router.
 *
 * rw4_slot_maps_create: encode one TMA tensor-map set per expert-cache slot (slot s holds an
 * expert's [N, K] RW4 weight at slot_packed[s] / slot_scale[s] / slot_zero[s]), once, when the
 * slots are allocated; nslots <= 80.  act = 1: stacked gate/up with the fused SwiGLU (as
 * rw4_moe_grouped).
 * rw4_moe_grouped_slots: rw4_moe_grouped where routed expert e's weight is the one in slot
 * slot_of[e] (DEVICE int32 [E], written by rw4_expert_residency); a routed expert without a valid
 * slot gets no output and sets RW4_DEVERR_SLOT (8) in the device status word.
 * rw4_expert_residency: one-thread kernel; from the permutation offsets (DEVICE int32 [E+1]) of
 * MoE layer `layer`, claim the slots of routed experts already resident, give each other routed
 * expert a free or least-recently-used slot not claimed in this call, and list those (copy_expert
 * / copy_slot int32 [E], ncopy int32 [1]).  State: where int32 [layers*E], owner int32 [S],
 * stamp int32 [S], clock int32 [1] (all initialised to -1 / -1 / 0 / 0 by the caller), counters
 * uint64 [2] (hits, fetches).
 * rw4_expert_residency_lfu: the same step under the reference's expert eviction, LFU with aging
 * (rocketllm/memory/cache.py:434-493), where rw4_expert_residency recycles least recently used:
 * routed experts in ascending order; a resident one is a hit; another takes a free slot, else the
 * slot of the resident expert with the smallest aged use count (ties: admitted first), never one
 * holding this layer's routed experts; then its use is counted and every aging_interval-th use
 * halves every count.  State (keys = layers*E >= (layer+1)*E): where int32 [keys] (-1), owner
 * int32 [S] (-1), uses double [keys] (0), admitted int32 [keys] (-1), state int64 [3] (0: uses
 * counted, experts admitted, agings), counters uint64 [2].  A routed expert that finds no slot
 * sets RW4_DEVERR_SLOT.
 * rw4_expert_residency_lfu_host: that step on HOST tables, on the calling thread (a host-routed
 * caller's form of the policy; the same compiled definition as the kernel's); RW4_EINVAL if a
 * routed expert finds no slot.
 * rw4_expert_copy: copy every listed expert's blob (host_blobs uint64 [layers*E]: DEVICE-visible
 * addresses of mapped pinned host blobs, each blob_bytes long) into its slot (slots + s *
 * slot_bytes); grid ctas_per_expert x E.
 * rw4_host_ptr_device: the device-visible address of pinned host memory, or an error for memory
 * that is not pinned and mapped (so a copy kernel is never given an address it cannot read).
 * ------------------------------------------------------------------------------------------- */
typedef struct rw4_slot_maps rw4_slot_maps;
int rw4_slot_maps_create(const uint8_t* const* slot_packed, const void* const* slot_scale,
                         const void* const* slot_zero, int32_t nslots, int64_t K, int64_t N,
                         int32_t act, rw4_slot_maps** out);
int rw4_slot_maps_destroy(rw4_slot_maps* maps);
int rw4_moe_grouped_slots(const void* x_perm_bf16, const int32_t* offsets, int32_t E,
                          int64_t max_rows, const rw4_slot_maps* maps, const int32_t* slot_of,
                          void* y_perm_bf16, void* stream);
int rw4_expert_residency(const int32_t* offsets, int32_t E, int32_t layer, int32_t* where,
                         int32_t* owner, int32_t* stamp, int32_t S, int32_t* clock,
                         int32_t* slot_of, int32_t* copy_expert, int32_t* copy_slot,
                         int32_t* ncopy, uint64_t* counters, void* stream);
int rw4_expert_residency_lfu(const int32_t* offsets, int32_t E, int32_t layer, int32_t keys,
                             int32_t* where, int32_t* owner, int32_t S, double* uses,
                             int32_t* admitted, int64_t* state, int64_t aging_interval,
                             int32_t* slot_of, int32_t* copy_expert, int32_t* copy_slot,
                             int32_t* ncopy, uint64_t* counters, void* stream);
int rw4_expert_residency_lfu_host(const int32_t* offsets, int32_t E, int32_t layer, int32_t keys,
                                  int32_t* where, int32_t* owner, int32_t S, double* uses,
                                  int32_t* admitted, int64_t* state, int64_t aging_interval,
                                  int32_t* slot_of, int32_t* copy_expert, int32_t* copy_slot,
                                  int32_t* ncopy, uint64_t* counters);
int rw4_expert_copy(const int32_t* copy_expert, const int32_t* copy_slot, const int32_t* ncopy,
                    int32_t layer, int32_t E, const uint64_t* host_blobs, int64_t blob_bytes,
                    uint8_t* slots, int64_t slot_bytes, int32_t S, int32_t ctas_per_expert,
                    void* stream);
int rw4_host_ptr_device(const void* host, void** device_ptr);

/* ---------------------------------------------------------------------------------------------
 * Decode attention over the int4 KV cache.  Replaces what the reference runs for one decode step
 * with its QuantizedKVCache (rocketllm/quant/kv_cache.py:277-316: every quantized block expanded
 * to the compute dtype, concatenated with the fp16 window, then the model's attention): softmax
 * attention of one query token straight over the packed history plus the window.
 *
 * Layout of each (batch, kv head) slot hs = b * kv_heads + kvh (all contiguous, 16-byte aligned):
 *   k_codes u8  [hs][groups_cap][head_dim][32]   group g, channel c: tokens 64g.. two per byte
 *   k_sz    f16 [hs][groups_cap][head_dim][2]    (scale, zero) per channel per group
 *   v_codes u8  [hs][groups_cap*64][head_dim/2]  per token, channels two per byte
 *   v_sz    f16 [hs][groups_cap*64][head_dim/64][2]  (scale, zero) per token per 64 channels
 *   k_res / v_res bf16 [hs][res_cap][head_dim]   the window, first res_len tokens valid
 * Codes and scales are the reference's quantize(K, axis=2, 64) / quantize(V, axis=3, 64) output
 * (value = code * scale + zero).  q bf16 [batch][heads][head_dim] with element strides
 * (q_stride_b, q_stride_h, 1); out bf16 likewise.  Query head h reads kv head h / (heads /
 * kv_heads).  head_dim 64 or 128, heads / kv_heads <= 16, groups + res_len >= 1.
 * ------------------------------------------------------------------------------------------- */
/* rw4_kv_attention: the same over q_len >= 1 query positions that are the window's LAST q_len
 * tokens (a speculative verify pass or a short chunk of one unpadded sequence per batch row):
 * position i attends to every quantized token and to the window's first res_len - q_len + 1 + i
 * tokens (causal).  q [batch][heads][q_len][head_dim] with element strides (q_stride_b,
 * q_stride_h, q_stride_q, 1), out likewise (out_stride_q for the position); q_len * heads /
 * kv_heads <= 16, q_len <= res_len. */
int rw4_kv_attention(const void* q, int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_q,
                     int32_t batch, int32_t heads, int32_t kv_heads, int32_t head_dim,
                     int32_t q_len, const uint8_t* k_codes, const void* k_sz,
                     const uint8_t* v_codes, const void* v_sz, int64_t groups_cap, int64_t groups,
                     const void* k_res, const void* v_res, int64_t res_cap, int64_t res_len,
                     float scaling, void* out, int64_t out_stride_b, int64_t out_stride_h,
                     int64_t out_stride_q, void* stream);
int rw4_kv_attention_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h, int32_t batch,
                            int32_t heads, int32_t kv_heads, int32_t head_dim,
                            const uint8_t* k_codes, const void* k_sz, const uint8_t* v_codes,
                            const void* v_sz, int64_t groups_cap, int64_t groups,
                            const void* k_res, const void* v_res, int64_t res_cap, int64_t res_len,
                            float scaling, void* out, int64_t out_stride_b, int64_t out_stride_h,
                            void* stream);

/* ---------------------------------------------------------------------------------------------
 * Streaming: pinned host staging pool + host->device transfer engine.
 *
 * rw4_pool_* replaces HostStagingPool (rocketllm/streaming/staging.py:80-273): pinned buffers in
 * power-of-two size classes (at least 2^16 bytes), leased, never handed to a second caller while
 * leased, allocated once and reused; a lease that would exceed the budget fails with RW4_EBUSY
 * (the Python shim then falls back to a transient buffer, as the reference does).
 *
 * rw4_xfer_* replaces WeightTransfer / TransferHandle (rocketllm/streaming/transfer.py:30-292):
 * each send is split into chunks issued round-robin on the engine's own copy streams (so two DMA
 * engines work on one layer), and gets a ticket whose completion is an event recorded behind all of
 * its chunks.  Compute waits on a ticket device-side (rw4_xfer_wait), never on the host.  A pooled
 * buffer must not be released before its ticket completes (rw4_xfer_query / rw4_xfer_sync).
 * ------------------------------------------------------------------------------------------- */

typedef struct rw4_pool rw4_pool;
typedef struct rw4_xfer rw4_xfer;

/* Pool with a pinned-byte budget (0 = no pinned buffers: every lease fails with RW4_EBUSY). */
int rw4_pool_create(size_t budget_bytes, rw4_pool** out);
int rw4_pool_destroy(rw4_pool* pool);
/* Lease a pinned buffer of at least `bytes` (smallest free buffer that fits; else a new one of the
 * size class if the budget allows; else RW4_EBUSY).  Returns its id and host address. */
int rw4_pool_lease(rw4_pool* pool, size_t bytes, int32_t* id, void** host);
int rw4_pool_release(rw4_pool* pool, int32_t id);
/* resident bytes, buffers, leased buffers, hits, misses */
int rw4_pool_stats(rw4_pool* pool, uint64_t* resident, int32_t* buffers, int32_t* leased,
                   uint64_t* hits, uint64_t* misses);

/* Transfer engine for `device` with `copy_streams` (1..8) non-blocking copy streams. */
int rw4_xfer_create(int32_t device, int32_t copy_streams, rw4_xfer** out);
int rw4_xfer_destroy(rw4_xfer* x);
/* Async H2D copy of n bytes host -> device, chunked (chunk_bytes = 0: one copy), after the copy
 * streams have waited for `after_stream`'s work so far when after_stream != NULL (used to keep a
 * reused device buffer from being overwritten while compute still reads it; pass cudaStreamLegacy,
 * (void*)1, to order after the legacy default stream).  *ticket identifies the send. */
int rw4_xfer_send(rw4_xfer* x, void* dst, const void* src, size_t n, size_t chunk_bytes,
                  void* after_stream, uint64_t* ticket);
/* Make `stream` wait device-side for the ticket's copies. */
int rw4_xfer_wait(rw4_xfer* x, uint64_t ticket, void* stream);
/* 1 if the ticket's copies completed, 0 if still in flight (never blocks). */
int rw4_xfer_query(rw4_xfer* x, uint64_t ticket);
/* Block until the ticket completes or timeout_ms passes (-1 = no limit): RW4_ETIMEOUT then. */
int rw4_xfer_sync(rw4_xfer* x, uint64_t ticket, int64_t timeout_ms);
/* Counters: sends, bytes, chunks, tickets still tracked. */
int rw4_xfer_stats(rw4_xfer* x, uint64_t* sends, uint64_t* bytes, uint64_t* chunks,
                   int32_t* in_flight);

/*
 * rw4_ring_*: a fixed ring of `slots` pinned staging slots of slot_bytes each in front of a
 * transfer engine with `copy_streams` copy streams on the current device -- the slot-ring form of
 * the pool + engine above, for callers that stage layer bytes from I/O worker threads.  Workers
 * fill a slot with rw4_ring_stage (a host memcpy; or read into the address from rw4_ring_slot);
 * the forward thread sends it with rw4_ring_submit (chunked over the copy streams; `done_event`,
 * a cudaEvent_t or NULL, is recorded behind the copies) and makes compute wait on the device with
 * rw4_ring_wait_compute (every slot's last submit).  A slot whose last submit is still in flight
 * is refused for staging and submitting (RW4_EBUSY): the reference's lease rule
 * (rocketllm/streaming/staging.py:33-66) per slot; a slot that rw4_ring_stage is still copying
 * into (another thread) is refused for submitting and for a second stage the same way.  The address
 * rw4_ring_slot returns is for a caller that owns the slot until it submits it (no stage into it
 * meanwhile).  rw4_ring_destroy waits for copies in flight.
 * slots 1..64, copy_streams 1..8.
 */
typedef struct rw4_ring rw4_ring;
int rw4_ring_create(size_t slot_bytes, int32_t slots, int32_t copy_streams, rw4_ring** out);
int rw4_ring_destroy(rw4_ring* ring);
int rw4_ring_slot(rw4_ring* ring, int32_t slot, void** host);
int rw4_ring_stage(rw4_ring* ring, int32_t slot, size_t offset, const void* src, size_t n);
int rw4_ring_submit(rw4_ring* ring, int32_t slot, void* dst, size_t n, void* done_event);
int rw4_ring_wait_compute(rw4_ring* ring, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RW4_H */
