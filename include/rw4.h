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
 * rw4_quantize: encode w[N, K] (dtype w_dtype: RW4_F32 or RW4_BF16) into packed/scale/zero,
 * bit-exact with quantize(w, axis=1, group_size=group) (rocketllm/quant/kv_cache.py:190-221),
 * including the bf16 scale arithmetic and the repeat-last-value padding of a ragged K.
 * Output rows have ceil(K/group) groups.
 */
int rw4_quantize(const void* w, int32_t w_dtype, int64_t N, int64_t K, int32_t group,
                 uint8_t* packed, void* scale_f16, void* zero_f16, void* stream);

/*
 * rw4_linear: y[M, N] = x[M, K] . W[N, K]^T, bf16 in and out, fp32 accumulation, W in RW4.
 * Replaces the nn.Linear / F.linear call a transformers module makes on a dequantized weight
 * (transformers models/llama/modeling_llama.py:171-184 via rocketllm/base.py:848-855).
 * M <= 16 runs the dequant-GEMV; larger M the tensor-core GEMM.  group must be 64 and K a
 * multiple of 64; x, y, packed, scale and zero must be 16-byte aligned.
 */
int rw4_linear(const void* x_bf16, int64_t M, int64_t K, const uint8_t* packed,
               const void* scale_f16, const void* zero_f16, int64_t N, int32_t group,
               void* y_bf16, void* stream);

/* Which kernel rw4_linear would launch for (M, K, N): 1 = GEMV, 2 = tcgen05 GEMM,
 * 3 = GEMV over 16-row slices. Negative on invalid shapes. Host-only, launches nothing. */
int rw4_linear_path(int64_t M, int64_t K, int64_t N);

/* Reads the library's device status word on the current device after the work queued on `stream`
 * (synchronises that stream): bit 1 = a bounded wait inside a kernel gave up (the kernel returned
 * early and its outputs are invalid), bit 2 = a tensor-memory allocation failed.  clear != 0 resets
 * the word.  No reference counterpart: the reference has no device kernels that can wait. */
int rw4_device_status(uint32_t* word, int32_t clear, void* stream);

/* ---------------------------------------------------------------------------------------------
 * MoE routed experts (transformers models/mixtral/modeling_mixtral.py:62-98, the experts forward
 * the reference streams; rocketllm/base.py:1375-1464 for its fused-row path).
 * ------------------------------------------------------------------------------------------- */

/*
 * rw4_moe_permute: stable counting sort of the T*k (token, slot) pairs by expert id.
 * topk_idx int64 [T, k] with ids in [0, E).  Writes perm int32 [T*k] (perm[row] = t*k + j, rows of
 * expert e are offsets[e]..offsets[e+1]-1 in increasing t*k+j order) and offsets int32 [E+1].
 * Out-of-range ids are counted in an error word and make the call return RW4_EINVAL on the next
 * rw4_moe_check_status (the kernel itself skips them).  E <= 1024.
 */
int rw4_moe_permute(const int64_t* topk_idx, int64_t T, int32_t k, int32_t E, int32_t* perm,
                    int32_t* offsets, void* stream);

/*
 * rw4_moe_gather: x_perm[row] = x[perm[row] / k] for row in [0, T*k), bf16 rows of H values.
 */
int rw4_moe_gather(const void* x_bf16, const int32_t* perm, int64_t T, int32_t k, int64_t H,
                   void* x_perm_bf16, void* stream);

/*
 * rw4_moe_grouped: y_perm[rows of e] = act(x_perm[rows of e] . W_e^T) for every expert e with at
 * least one routed row; experts with none are never read.  Weights are per-expert RW4 tensors
 * given as device arrays of device pointers (packed_e[E], scale_e[E], zero_e[E]), each W_e of
 * shape [N, K].  `offsets` is the device int32 [E+1] from rw4_moe_permute; `max_rows` is an upper
 * bound on any expert's row count (T*k is always safe).
 * act = 0: plain linear (y_perm [T*k, N]).
 * act = 1: SwiGLU over a stacked gate/up weight of N = 2*I rows: y_perm[r, i] =
 *          silu(g) * u with g = bf16(x.W[i]), u = bf16(x.W[I+i]); y_perm is [T*k, I].
 */
int rw4_moe_grouped(const void* x_perm_bf16, const int32_t* offsets, int32_t E, int64_t max_rows,
                    const uint8_t* const* packed_e, const void* const* scale_e,
                    const void* const* zero_e, int64_t K, int64_t N, int32_t group, int32_t act,
                    void* y_perm_bf16, void* stream);

/*
 * rw4_moe_combine: out[t] = bf16( sum_{j<k} w[t, j] * y_perm[inv(t*k+j)] ), fp32 accumulation in
 * slot order j = 0..k-1 (deterministic, no atomics).  topk_w is fp32 [T, k] (w_dtype RW4_F32) or
 * bf16 (RW4_BF16); y_perm bf16 [T*k, H]; out bf16 [T, H].
 */
int rw4_moe_combine(const void* y_perm_bf16, const int32_t* perm, const void* topk_w,
                    int32_t w_dtype, int64_t T, int32_t k, int64_t H, void* out_bf16,
                    void* stream);

/* ---------------------------------------------------------------------------------------------
 * Host->device staging ring (rocketllm/streaming/staging.py:80-273 HostStagingPool.lease and
 * rocketllm/streaming/transfer.py:124-292 WeightTransfer.send_buffer / TransferHandle.resolve).
 * A ring owns `slots` pinned host buffers of `slot_bytes` each and `copy_streams` CUDA streams.
 * ------------------------------------------------------------------------------------------- */

typedef struct rw4_ring rw4_ring;

int rw4_ring_create(size_t slot_bytes, int32_t slots, int32_t copy_streams, int32_t device,
                    rw4_ring** out);
int rw4_ring_destroy(rw4_ring* ring);

/* Lease a free slot (blocking up to timeout_ms for an in-flight one to complete; -1 = forever).
 * Returns the slot index in *slot and its host pointer in *host. RW4_ETIMEOUT if none frees. */
int rw4_ring_acquire(rw4_ring* ring, int64_t timeout_ms, int32_t* slot, void** host);

/* Copy `n` bytes from host memory `src` into slot `slot` at byte `offset` (host memcpy on the
 * calling thread; io workers may call this). */
int rw4_ring_stage(rw4_ring* ring, int32_t slot, size_t offset, const void* src, size_t n);

/* Issue the H2D copy of bytes [0, n) of `slot` to device `dst`, split into chunks of
 * chunk_bytes (0 = one copy) spread round-robin over the ring's copy streams, and record the
 * slot's completion event.  The slot stays leased until that event fires. */
int rw4_ring_submit(rw4_ring* ring, int32_t slot, void* dst, size_t n, size_t chunk_bytes);

/* Make `stream` wait (device-side) for slot `slot`'s copies; never blocks the host. */
int rw4_ring_wait(rw4_ring* ring, int32_t slot, void* stream);

/* Release a slot once its copy has completed: returns 1 if released, 0 if still in flight
 * (non-blocking), and blocks up to timeout_ms when block != 0 (RW4_ETIMEOUT if it does not
 * complete in time). */
int rw4_ring_release(rw4_ring* ring, int32_t slot, int32_t block, int64_t timeout_ms);

/* Counters: bytes submitted, copies issued, acquire stalls, slots in flight. */
int rw4_ring_stats(rw4_ring* ring, uint64_t* bytes, uint64_t* copies, uint64_t* stalls,
                   int32_t* in_flight);

#ifdef __cplusplus
}
#endif

#endif /* RW4_H */
