/*
 * riallm_cuda.h -- C ABI of libriallm_cuda.so, the B200 (sm_100a) engine for
 * riallm's mixture-of-experts block forward with block-quantized weights.
 *
 * Plain pointers and sizes only: no C++ or torch types cross this boundary.
 * Every function returns riallm_status (0 = ok) unless it returns a size.
 * Device pointers are caller-owned unless a function says it allocates; the
 * library never frees caller memory. All work is asynchronous on the given
 * CUDA stream (a cudaStream_t passed as void*, NULL = legacy default stream).
 * One context per device per host thread.
 *
 * The reference (riallm, Rust) has no FFI of its own: each entry point below
 * names the reference function it stands in for (file:line inside the
 * riallm crate). A Rust `riallm-cuda` crate binds these with `extern "C"`.
 */
#ifndef RIALLM_CUDA_H
#define RIALLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RIALLM_CUDA_ABI_VERSION 1

/* Status codes. 1-4 map onto RiallmError variants (src/error.rs:8-47). */
typedef enum riallm_status {
  RIALLM_OK = 0,
  RIALLM_ERR_MEMORY = 1,        /* RiallmError::Memory */
  RIALLM_ERR_QUANTIZATION = 2,  /* RiallmError::Quantization */
  RIALLM_ERR_CONFIG = 3,        /* RiallmError::Config */
  RIALLM_ERR_MODEL_LOADING = 4, /* RiallmError::ModelLoading ("Tensor not found") */
  RIALLM_ERR_CUDA = 5,          /* device/runtime failure (RiallmError::Candle's role) */
  RIALLM_ERR_TIMEOUT = 6,       /* a bounded device-side wait expired */
  RIALLM_ERR_INVALID = 7        /* NULL or malformed argument */
} riallm_status;

/* CompressionType, src/config.rs:323-332. */
typedef enum riallm_compression {
  RIALLM_COMPRESSION_NONE = 0,     /* data is float32[numel] */
  RIALLM_COMPRESSION_FOUR_BIT = 1, /* NF4, 64-element blocks, 2 codes per byte */
  RIALLM_COMPRESSION_EIGHT_BIT = 2 /* 8-bit affine, 128-element blocks */
} riallm_compression;

typedef enum riallm_dtype {
  RIALLM_DTYPE_F32 = 0,
  RIALLM_DTYPE_BF16 = 1
} riallm_dtype;

/* Dequantization semantics.
 * REFERENCE: exactly src/quantization.rs:45-95 ((code - zero) * scale; an
 *   NF4 element at position 63 of its block uses the next block's scale and
 *   zero, and the tensor's last element falls back to scale 1, zero 0).
 * CODEBOOK: NF4 table[code] * scale (the intended NF4 decode); for 8-bit,
 *   code * scale + zero (the inverse of the quantizer). */
typedef enum riallm_dequant_mode {
  RIALLM_DEQUANT_REFERENCE = 0,
  RIALLM_DEQUANT_CODEBOOK = 1
} riallm_dequant_mode;

/* QuantizedTensor, src/quantization.rs:12-30, as device pointers. The
 * tensor's elements run over the flattened shape. */
typedef struct riallm_qtensor {
  int32_t qtype;             /* riallm_compression */
  int32_t block_size;        /* 64 (FOUR_BIT) or 128 (EIGHT_BIT) */
  const void* data;          /* packed codes, or float32 when qtype == NONE */
  const float* scales;       /* scales.len() == n_scales */
  const float* zero_points;  /* zero_points.len() == n_zero_points */
  uint64_t numel;            /* shape.iter().product() */
  uint64_t n_scales;
  uint64_t n_zero_points;
} riallm_qtensor;

/* One layer's MoE tensors (names as src/model.rs:762,791-792,825-831). */
typedef struct riallm_moe_weights {
  riallm_qtensor gate;               /* mlp.gate.weight            [E, H]     */
  riallm_qtensor gate_up_proj;       /* mlp.experts.gate_up_proj   [E, 2I, H] */
  riallm_qtensor down_proj;          /* mlp.experts.down_proj      [E, H, I]  */
  /* Optional Qwen3.5 shared expert; leave data == NULL when absent. */
  riallm_qtensor shared_gate_proj;   /* [Is, H] */
  riallm_qtensor shared_up_proj;     /* [Is, H] */
  riallm_qtensor shared_down_proj;   /* [H, Is] */
  riallm_qtensor shared_expert_gate; /* [1, H]  */
  int32_t shared_intermediate;       /* Is */
} riallm_moe_weights;

typedef struct riallm_ctx riallm_ctx;

/* ----------------------------------------------------------- context */

int32_t riallm_cuda_abi_version(void);

/* Creates a context on CUDA device `device` (DeviceSpec::Cuda(id),
 * src/config.rs:350-372; src/model.rs:100-104 picks the device). */
int32_t riallm_cuda_ctx_create(int32_t device, riallm_ctx** out);
int32_t riallm_cuda_ctx_destroy(riallm_ctx* ctx);

/* Message of the last failure on this context ("" when none). */
const char* riallm_cuda_last_error(const riallm_ctx* ctx);

/* ------------------------------------------------------------ memory
 * src/memory.rs:60-78 (get_memory_stats), :113-125 (move_tensors_to_device),
 * :183-198 (synchronize_device). */

int32_t riallm_cuda_alloc(riallm_ctx* ctx, uint64_t bytes, void** dptr);
int32_t riallm_cuda_free(riallm_ctx* ctx, void* dptr);
int32_t riallm_cuda_host_alloc_pinned(riallm_ctx* ctx, uint64_t bytes, void** hptr);
int32_t riallm_cuda_host_free_pinned(riallm_ctx* ctx, void* hptr);
int32_t riallm_cuda_memcpy_h2d_async(riallm_ctx* ctx, void* dst, const void* src,
                                     uint64_t bytes, void* stream);
int32_t riallm_cuda_memcpy_d2h_async(riallm_ctx* ctx, void* dst, const void* src,
                                     uint64_t bytes, void* stream);
/* Waits for `stream`; returns RIALLM_ERR_TIMEOUT (and clears the record and
 * the scratch arena's call counters, so the context stays usable) when a
 * kernel of this context aborted because a bounded device-side wait
 * expired. riallm reports failures only as Result<_, RiallmError>
 * (src/error.rs:8-47); it has no device-side failure of this kind. */
int32_t riallm_cuda_stream_synchronize(riallm_ctx* ctx, void* stream);

/* No counterpart in the reference. Bound, in ns, of a kernel's wait for
 * work that other CTAs of the same launch publish (the expert GEMM's
 * split-tile owner waiting for partial sums). 0 restores the default of 1 s;
 * other values must be >= 1000. Waits inside a CTA (its own pipeline) keep
 * the 1 s bound. */
int32_t riallm_cuda_ctx_set_wait_limit(riallm_ctx* ctx, uint64_t wait_ns);

/* No counterpart in the reference; a test hook for the timeout path. In the
 * next riallm_cuda_moe_forward call of this context, every expert-GEMM tile
 * that is split across CTAs is finished by a CTA that waits for a partial-sum
 * count no CTA reaches, so its bounded wait expires: that CTA stops, the
 * call's output is undefined, and riallm_cuda_stream_synchronize returns
 * RIALLM_ERR_TIMEOUT. Nothing faults or hangs; later calls are unaffected. */
int32_t riallm_cuda_ctx_expire_next_wait(riallm_ctx* ctx);
int32_t riallm_cuda_memory_stats(riallm_ctx* ctx, uint64_t* free_bytes,
                                 uint64_t* total_bytes);

/* ---------------------------------------------------- layer streaming */

/* Stands in for the per-forward device moves of a streamed layer
 * (load_layer_to_device, src/model.rs:1131-1201; move_tensors_to_device,
 * src/memory.rs:113-125) and acts on ModelOptions::prefetch_layers /
 * prefetch_buffer_size (src/config.rs:389-393), which riallm leaves unused.
 * A streamer holds `depth` device slots of `slot_bytes` (a multiple of 256)
 * and a copy stream. device_slots is a caller buffer of depth * slot_bytes
 * bytes (256-byte aligned), or NULL to allocate one. */
typedef struct riallm_streamer riallm_streamer;
int32_t riallm_cuda_streamer_create(riallm_ctx* ctx, int32_t depth, uint64_t slot_bytes,
                                    void* device_slots, riallm_streamer** out);
int32_t riallm_cuda_streamer_destroy(riallm_streamer* s);
/* Copies `bytes` of a layer's packed weights from host_src (pinned host
 * memory, or the copy is not asynchronous) into slot layer % depth on the
 * copy stream, after the compute that last used the slot released it.
 * RIALLM_ERR_CONFIG if that slot still holds an unreleased layer (prefetch
 * at most depth layers ahead); RIALLM_ERR_MEMORY if bytes > slot_bytes. */
int32_t riallm_cuda_streamer_prefetch(riallm_streamer* s, int32_t layer, const void* host_src,
                                      uint64_t bytes);
/* The same for n byte ranges of the layer's blob, [offsets[i], offsets[i] +
 * sizes[i]), each copied to the same offset of the slot (one ready event
 * for all): a decode step copies only the experts its batch routes to. The
 * bytes outside the ranges keep whatever the slot held. RIALLM_ERR_MEMORY
 * if a range leaves the slot. */
int32_t riallm_cuda_streamer_prefetch_ranges(riallm_streamer* s, int32_t layer, const void* host_src,
                                             const uint64_t* offsets, const uint64_t* sizes, int32_t n);
/* Makes `stream` wait for the layer's copy and returns its device address. */
int32_t riallm_cuda_streamer_acquire(riallm_streamer* s, int32_t layer, void* stream, void** dptr);
/* Marks the end of the layer's use on `stream` (after its last kernel). */
int32_t riallm_cuda_streamer_release(riallm_streamer* s, int32_t layer, void* stream);
/* Totals so far: bytes copied, copies, and the copies' device time (ms).
 * Waits for the copy stream. */
int32_t riallm_cuda_streamer_stats(riallm_streamer* s, uint64_t* bytes, uint64_t* copies,
                                   double* copy_ms);

/* ------------------------------------------------------ quantization */

/* Number of scale/zero blocks and packed data bytes for numel elements. */
uint64_t riallm_quant_num_blocks(int32_t qtype, uint64_t numel);
uint64_t riallm_quant_data_bytes(int32_t qtype, uint64_t numel);

/* quantize_tensor (src/quantization.rs:99-107 -> :111-176 NF4,
 * :199-245 8-bit), bit-identical to the reference's host loops.
 * src: float32[numel] on the device; outputs sized by the helpers above. */
int32_t riallm_cuda_quantize(riallm_ctx* ctx, int32_t qtype, const float* src,
                             uint64_t numel, uint8_t* data, float* scales,
                             float* zero_points, void* stream);

/* QuantizedTensor::dequantize (src/quantization.rs:34-95). dst holds numel
 * values of dst_dtype (bf16 values are the float32 results rounded to
 * nearest even). NF4 requires data length ceil(numel/2). */
int32_t riallm_cuda_dequantize(riallm_ctx* ctx, const riallm_qtensor* t,
                               int32_t mode, void* dst, int32_t dst_dtype,
                               void* stream);

/* --------------------------------------------------------- MoE block */

#define RIALLM_MOE_ADD_TO_OUT 1u /* out += block(x) instead of out = block(x) */

/* apply_qwen3_5_moe (src/model.rs:751-818, shared expert :820-834):
 * router matmul -> softmax -> stable top-k -> renormalise -> per-expert
 * SwiGLU (gate = rows [0,I) of gate_up_proj[e], up = rows [I,2I)) -> down
 * projection -> routing-weight scale -> sum in expert-ascending order
 * (+ shared expert). x and out are [T,H] in act_dtype. Expert tensors must be
 * FOUR_BIT or EIGHT_BIT; gate/shared tensors may be any compression.
 * Shape limits: H % 256 == 0, I % 256 == 0, E <= 256, k <= 16, k <= E.
 * Scratch comes from the context's device arena, which grows with
 * cudaMalloc on demand (see riallm_cuda_moe_reserve). Calls of one context
 * share that arena: issue them on one stream (or order them). */
int32_t riallm_cuda_moe_forward(riallm_ctx* ctx, const riallm_moe_weights* w,
                                const void* x, void* out, int32_t T, int32_t H,
                                int32_t I, int32_t E, int32_t k,
                                int32_t act_dtype, uint32_t flags, void* stream);

/* No counterpart in the reference (it has no multi-GPU path). One rank's
 * share of an expert-parallel MoE block: rank r of W owns the experts
 * [e_begin, e_begin + e_local). x holds the bf16 tokens of every rank
 * ([T,H], gathered by the caller), w->gate the full router [E,H], and
 * w->gate_up_proj / w->down_proj only the owned experts ([e_local,2I,H] and
 * [e_local,H,I]). Every token is routed over all E experts exactly as by
 * riallm_cuda_moe_forward; partial [T,H] (float32) receives, per token, the
 * routing-weighted sum of its owned experts' outputs in expert-ascending
 * order (0 where it has none). Summing the W partials (a reduce-scatter)
 * and rounding to bf16 gives riallm_cuda_moe_forward's output up to float32
 * summation order inside the expert GEMMs (their K ranges are split across
 * SMs differently when a rank holds fewer experts). Routed experts only. */
int32_t riallm_cuda_moe_forward_ep(riallm_ctx* ctx, const riallm_moe_weights* w,
                                   const void* x, float* partial, int32_t T,
                                   int32_t H, int32_t I, int32_t E, int32_t k,
                                   int32_t e_begin, int32_t e_local, void* stream);

/* Grows the context's scratch arena for blocks up to these sizes now, so
 * that later riallm_cuda_moe_forward calls allocate nothing (and can be
 * captured in a CUDA graph). An arena outgrown by a later, larger call is
 * kept until the context is destroyed, so graphs that captured earlier calls
 * stay valid. */
int32_t riallm_cuda_moe_reserve(riallm_ctx* ctx, int32_t T, int32_t H, int32_t I,
                                int32_t E, int32_t k, int32_t act_dtype);

/* Router and bucketing only (src/model.rs:762-789), for bit-exact checks.
 * topk_idx/topk_w [T,k]; counts [E]; offsets [E+1]; perm_pair [T*k]
 * (pair ids t*k+j grouped by expert ascending, token-ascending within an
 * expert). Any output except topk_idx may be NULL. */
int32_t riallm_cuda_moe_route(riallm_ctx* ctx, const riallm_qtensor* gate,
                              const void* x, int32_t T, int32_t H, int32_t E,
                              int32_t k, int32_t act_dtype, int32_t* topk_idx,
                              float* topk_w, int32_t* counts, int32_t* offsets,
                              int32_t* perm_pair, void* stream);

/* No counterpart in the reference. The MoE block for callers that cannot
 * allocate device memory: code whose host owns all device memory, or that
 * must not call cudaMalloc (it can synchronize the device and has no bounded
 * latency), and so can neither create a riallm_ctx nor let the library grow
 * its scratch arena. The caller passes weights, x and out; all scratch comes
 * from one 24 MiB array compiled into the library, which every GPU that
 * loads the library holds until the process exits. Nothing is allocated.
 * Limits: bf16 x/out ([T,H], 16-byte aligned), routed experts only (no
 * shared expert), the same shape rules and argument checks (with the same
 * status codes) as riallm_cuda_moe_forward, and the call's scratch layout
 * must fit 24 MiB (for hidden 4096 / intermediate 14336, up to 472
 * token-expert pairs, T*k); larger calls return RIALLM_ERR_MEMORY without
 * launching anything. The first call on each device looks up the array's
 * device address (and sets kernel attributes); make that first call before
 * any stream capture (a look-up that fails is retried by the next call).
 * Every call reuses the same array and leaves its contents behind (the
 * counters that must start at zero are cleared at the start of every call),
 * so calls that overlap on the GPU (other streams or host threads) race on
 * it: serialize them. Runs on the current CUDA device and on `stream`. A
 * RIALLM_OK return means the work was queued; whether it completed cleanly
 * is reported by riallm_cuda_moe_forward_noalloc_sync. */
int32_t riallm_cuda_moe_forward_noalloc(const riallm_moe_weights* w, const void* x,
                                        void* out, int32_t T, int32_t H, int32_t I,
                                        int32_t E, int32_t k, uint32_t flags,
                                        void* stream);

/* No counterpart in the reference. Waits for `stream`, then reports whether
 * every riallm_cuda_moe_forward_noalloc call on the current device since the
 * last report ran to completion: RIALLM_OK, or RIALLM_ERR_TIMEOUT when a
 * bounded device-side wait expired in one of them (the `out` of such a call
 * is undefined). The record is cleared by reading it. Allocates nothing. */
int32_t riallm_cuda_moe_forward_noalloc_sync(void* stream);

/* ---------------------------------------------------------- profiling
 * The reference's Profiler (src/profiler.rs:75-96) times each layer on the
 * host wall clock. Here, when enabled, riallm_cuda_moe_forward records a
 * CUDA event pair around each phase on the call's stream; reading
 * synchronizes, returns the accumulated device milliseconds per phase since
 * the last read, and resets them. The launch counter counts every kernel
 * this context has launched (never reset). */
typedef enum riallm_phase {
  RIALLM_PHASE_ROUTE = 0,    /* router weight decode + router + permutation */
  RIALLM_PHASE_GATHER = 1,   /* token rows into expert order */
  RIALLM_PHASE_GATE_UP = 2,  /* expert gate/up GEMM + SwiGLU */
  RIALLM_PHASE_DOWN = 3,     /* expert down GEMM */
  RIALLM_PHASE_SHARED = 4,   /* shared expert */
  RIALLM_PHASE_COMBINE = 5,  /* weighted combine */
  RIALLM_PHASE_DISPATCH = 6, /* expert parallel: token rows to the experts' ranks */
  RIALLM_PHASE_RETURN = 7,   /* expert parallel: expert outputs back to the tokens' ranks */
  RIALLM_NUM_PHASES = 8
} riallm_phase;

/* ------------------------------------------------ expert parallelism
 * No counterpart in the reference (riallm runs every layer on one device,
 * src/model.rs:231-258). Ranks of one node, one context per GPU: rank r of
 * W owns experts [r E/W, (r+1) E/W). The library opens NCCL at run time
 * (libnccl.so.2) and keeps one communicator per context. */

/* A fresh 128-byte NCCL unique id (ncclUniqueId); rank 0 makes it and the
 * caller hands it to every rank over its own channel.
 * RIALLM_ERR_CONFIG if NCCL cannot be loaded. */
int32_t riallm_cuda_ep_unique_id(uint8_t* unique_id_out);
/* Joins the W ranks' communicator (collective: every rank calls it with the
 * same id). */
int32_t riallm_cuda_ep_init(riallm_ctx* ctx, const uint8_t* unique_id, int32_t rank, int32_t world);
/* Leaves it (also done by riallm_cuda_ctx_destroy). */
int32_t riallm_cuda_ep_destroy(riallm_ctx* ctx);
/* RIALLM_OK, or RIALLM_ERR_CUDA with the message when NCCL reports an
 * asynchronous error on the communicator (a peer died or a link failed):
 * a host watchdog polls it between steps. */
int32_t riallm_cuda_ep_async_error(riallm_ctx* ctx);

/* The expert-parallel MoE block (apply_qwen3_5_moe, src/model.rs:751-818,
 * split over the ranks): x and out are this rank's [T, H] bf16 tokens;
 * w->gate is the full router [E, H], w->gate_up_proj / w->down_proj hold
 * only this rank's experts ([E/W, 2I, H], [E/W, H, I];
 * QuantizedTensor::expert_slice). Every rank calls it with the same T >= 1
 * and shape. Each rank routes its own tokens over all E experts, sends the
 * token rows of every pair to the rank owning the pair's expert (NCCL
 * point-to-point, one message per peer each way), runs its experts on what
 * it received, sends the outputs back, and sums each token's pairs in
 * expert-ascending order with the routing weights, as riallm_cuda_moe_forward
 * does (outputs equal up to float32 summation order inside the expert
 * GEMMs). The exchange sizes are copied to the host once per call (a
 * synchronization of `stream`), so a call cannot be captured in a CUDA
 * graph. The receive buffers live in a second arena of the context, sized
 * by the rows the call receives and grown with cudaMalloc when a call
 * receives more. Routed experts only. */
int32_t riallm_cuda_moe_forward_ep_a2a(riallm_ctx* ctx, const riallm_moe_weights* w, const void* x,
                                       void* out, int32_t T, int32_t H, int32_t I, int32_t E, int32_t k,
                                       uint32_t flags, void* stream);

/* Peer-memory transport for the same block (collective: every rank calls
 * it after riallm_cuda_ep_init, with the same arguments). Allocates this
 * rank's symmetric buffer for calls of up to max_tokens tokens of this
 * shape (flags, the rows it can receive, its pairs' returned rows), maps
 * every peer's through CUDA IPC (handles exchanged over the communicator)
 * and the local plan and expert buffers. Calling it again replaces the
 * set-up; riallm_cuda_ep_destroy frees it. */
int32_t riallm_cuda_ep_peer_init(riallm_ctx* ctx, int32_t max_tokens, int32_t H, int32_t I, int32_t E, int32_t k);
/* riallm_cuda_moe_forward_ep_a2a's block over the peer-memory transport:
 * the pair counts are all-gathered on the device (NCCL), each pair row is
 * stored straight into its expert's rank's receive area and each output row
 * into its token's rank's return area by the library's kernels (plain
 * stores to mapped peer memory over NVLink), and the ranks hand the buffers
 * back and forth with epoch flags (bounded waits: RIALLM_ERR_TIMEOUT through
 * riallm_cuda_stream_synchronize). No host synchronisation, so a call can
 * be captured in a CUDA graph. T <= max_tokens (ranks may differ); the
 * shape must be riallm_cuda_ep_peer_init's. Routed experts only. */
int32_t riallm_cuda_moe_forward_ep_peer(riallm_ctx* ctx, const riallm_moe_weights* w, const void* x,
                                        void* out, int32_t T, int32_t H, int32_t I, int32_t E, int32_t k,
                                        uint32_t flags, void* stream);

/* Host-only helper of the exchange above (no device work): from the pair
 * counts each rank sends to this rank, recv_counts[s * e_local + e] (rank s,
 * local expert e), where the received rows go: expert_counts[e],
 * expert_offsets[e] (e_local + 1 entries, expert-major) and
 * block_pos[s * e_local + e] (first row of rank s's rows for expert e). */
int32_t riallm_ep_exchange_plan(int32_t world, int32_t e_local, const int32_t* recv_counts,
                                int32_t* expert_counts, int32_t* expert_offsets, int32_t* block_pos);

/* ------------------------------------------------------------ events
 * Ordering between the caller's streams (riallm has no streams; its device
 * work is synchronous). Events are created without timing. */
int32_t riallm_cuda_event_create(riallm_ctx* ctx, void** event_out);
int32_t riallm_cuda_event_destroy(riallm_ctx* ctx, void* event);
int32_t riallm_cuda_event_record(riallm_ctx* ctx, void* event, void* stream);
/* Makes `stream` wait for the event's last record (no host blocking). */
int32_t riallm_cuda_stream_wait_event(riallm_ctx* ctx, void* stream, void* event);
int32_t riallm_cuda_event_synchronize(riallm_ctx* ctx, void* event);

/* ---------------------------------------------------------- decoder layer
 * The dense parts of a decoder layer around the MoE block, for end-to-end
 * decoding with a device-resident bf16 KV cache. riallm runs these through
 * candle on each forward (src/model.rs:456-468, 912-1071, 1317-1328).
 * Activations are bf16 (RIALLM_DTYPE_BF16 layout), arithmetic float32.
 * Positions are a device int32 array pos[B]: row b*T + t of a call holds the
 * token at position pos[b] + t, so one decode step can be graph-replayed
 * while pos advances on the device. */

/* RMSNorm, src/model.rs:456-468: out = bf16(x * rsqrt(mean(x^2) + eps) * w)
 * per row of x [rows, H]. With delta != NULL the residual add
 * x = bf16(x + delta) is stored back to x first. w is float32 [H].
 * H % 8 == 0; x, delta and out 16-byte aligned. */
int32_t riallm_cuda_rmsnorm(riallm_ctx* ctx, void* x, const void* delta, const float* w,
                            void* out, int32_t rows, int32_t H, float eps, void* stream);

/* Rotary embedding, src/model.rs:1002-1071 (rotate-half, angle =
 * float(position) * inv_freq[i], i < d/2), of the q and k heads of
 * qkv [B*T, (nh + 2*nkv) * d] (q heads, k heads, v heads). Rotated q goes to
 * q_out [B*T, nh*d]; rotated k and the v heads are written into the caches
 * [B, nkv, S_max, d] at each row's position. Positions outside [0, S_max)
 * write nothing to the caches. */
int32_t riallm_cuda_rope_kv_append(riallm_ctx* ctx, const void* qkv, const int32_t* pos,
                                   int32_t B, int32_t T, int32_t nh, int32_t nkv, int32_t d,
                                   const float* inv_freq, void* q_out, void* k_cache,
                                   void* v_cache, int32_t S_max, void* stream);

/* Causal grouped-query attention over the cache, src/model.rs:912-1000 with
 * the query heads h of KV head h / (nh/nkv) (repeat_heads,
 * src/model.rs:1317-1328): row b*T + t attends cache positions
 * [0, pos[b] + t] (clamped to S_max) with scores q.k / sqrt(d), a softmax
 * and the weighted sum of v, all float32. q and out are [B*T, nh*d].
 * d is 64 or 128; nh / nkv is 1, 2, 4, 6 or 8. When the (sequence, kv head,
 * token) groups are too few to fill the GPU, each group's keys are split
 * over several CTAs that merge through a workspace owned by the context:
 * calls of one context must not overlap (issue them on one stream). */
int32_t riallm_cuda_attention(riallm_ctx* ctx, const void* q, const void* k_cache,
                              const void* v_cache, const int32_t* pos, int32_t B, int32_t T,
                              int32_t nh, int32_t nkv, int32_t d, int32_t S_max, void* out,
                              void* stream);

/* y = bf16(x · wᵀ) with float32 accumulation for decode-sized batches: x
 * [M, K], w [N, K] (a projection weight, e.g. q/k/v, o or the LM head,
 * src/model.rs:912-940), y [M, N], all bf16; M <= 8, K % 256 == 0, x and w
 * 16-byte aligned. The weight is streamed once. */
int32_t riallm_cuda_linear_bf16(riallm_ctx* ctx, const void* x, const void* w, void* y, int32_t M,
                                int32_t N, int32_t K, void* stream);

int32_t riallm_cuda_profile_enable(riallm_ctx* ctx, int32_t enable);
int32_t riallm_cuda_profile_read(riallm_ctx* ctx, float* ms_per_phase,
                                 uint64_t* calls);
uint64_t riallm_cuda_launch_count(const riallm_ctx* ctx);

#ifdef __cplusplus
}
#endif
#endif /* RIALLM_CUDA_H */
