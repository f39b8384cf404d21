/*
 * riallm_oracle.h -- CPU restatement of riallm's block quantization and
 * mixture-of-experts block forward.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product (riallm_b200/, the CUDA
 * library, bench.py's GPU arms) links or calls this code; only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm use it,
 * and only as the parity reference or as the timed CPU port.
 *
 * PARITY UNPINNED: the reference is Rust (candle 0.8) and cannot be built or
 * run in this environment (no cargo/rustc, no network), and its own tests
 * (tests/integration_test.rs:124-148) assert only qtype, shape and
 * non-empty scales. The restatement is pinned against hand-derived known
 * answers computed from the reference source on the reference's own test
 * inputs (tests/test_oracle_pins.py) and cross-checked by an independent
 * numpy mirror (oracle/oracle.py).
 *
 * Reference files followed (paths inside the riallm crate):
 *   src/quantization.rs:45-76    dequantize_4bit  (NF4, incl. block-end quirk)
 *   src/quantization.rs:79-95    dequantize_8bit
 *   src/quantization.rs:111-196  quantize_4bit_nf4 + normalize_and_quantize_nf4
 *   src/quantization.rs:199-245  quantize_8bit_blockwise
 *   src/model.rs:751-818         apply_qwen3_5_moe (router, bucketing, experts)
 *   src/model.rs:820-834         apply_qwen3_5_shared_expert
 */
#ifndef RIALLM_ORACLE_H
#define RIALLM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { RO_NONE = 0, RO_FOUR_BIT = 1, RO_EIGHT_BIT = 2 };

/* One tensor in the reference's QuantizedTensor layout
 * (src/quantization.rs:12-30). For RO_NONE, data is float32[numel]. */
typedef struct ro_qtensor {
  int32_t qtype;
  int32_t block_size;
  const void* data;
  const float* scales;
  const float* zero_points;
  uint64_t numel;
  uint64_t n_scales;      /* scales.len() */
  uint64_t n_zero_points; /* zero_points.len() */
} ro_qtensor;

/* Sizes of the quantized outputs for n elements. */
uint64_t ro_num_blocks(int32_t qtype, uint64_t n);
uint64_t ro_data_bytes(int32_t qtype, uint64_t n);

/* src/quantization.rs:111-196. Writes ro_data_bytes bytes and ro_num_blocks
 * scales / zero points. */
void ro_quantize_nf4(const float* v, uint64_t n, uint8_t* data, float* scales,
                     float* zeros);
/* src/quantization.rs:199-245. */
void ro_quantize_int8(const float* v, uint64_t n, uint8_t* data, float* scales,
                      float* zeros);

/* src/quantization.rs:45-76, literal loop (running scale index).
 * Returns the number of values written to out. */
uint64_t ro_dequantize_nf4(const uint8_t* data, uint64_t n_bytes,
                           const float* scales, uint64_t n_scales,
                           const float* zeros, uint64_t n_zeros,
                           uint64_t numel, uint64_t block_size, float* out);
/* src/quantization.rs:79-95. Returns values written (== n_bytes). */
uint64_t ro_dequantize_int8(const uint8_t* data, uint64_t n_bytes,
                            const float* scales, uint64_t n_scales,
                            const float* zeros, uint64_t n_zeros,
                            uint64_t block_size, float* out);

/* Elements [start, start+len) of a tensor as float32, using the closed form
 * of the reference's scale index (element e of an NF4 tensor uses block
 * (e+1)/block_size; int8 uses e/block_size). bf16_round != 0 rounds each
 * value to bfloat16 (round to nearest even), as the bf16 activation mode does. */
void ro_tensor_span_f32(const ro_qtensor* t, uint64_t start, uint64_t len,
                        int32_t bf16_round, float* out);

/* Own exponential (Cody-Waite reduction + degree-7 Taylor polynomial), shared
 * bit-for-bit with the CUDA router so that routing is reproducible. */
float ro_expf(float x);

/* Router, src/model.rs:762-770, with a fixed fp32 reduction order:
 * logits[t,e] = sum over 32 lane partials; lane l accumulates the 8-element
 * chunks c = l, l+32, ... with fused multiply-adds, then a xor butterfly
 * (offsets 16,8,4,2,1) adds the lanes. softmax: max, ro_expf(l-max),
 * sequential sum over e, IEEE division. top-k: stable descending (ties to the
 * lower index). renorm: divide by the sequential sum of the k picked probs.
 * x is bf16 (x_bf16 != 0, uint16 bits) or float32, row-major [T,H];
 * wg is float32 [E,H]. Any of logits/probs may be NULL. */
void ro_router(const void* x, int32_t x_bf16, int32_t T, int32_t H,
               const float* wg, int32_t E, int32_t k, float* logits,
               float* probs, int32_t* topk_idx, float* topk_w);

/* Host bucketing, src/model.rs:776-789, as a counting sort.
 * counts[E], offsets[E+1]; perm_pair[T*k] lists pair ids (t*k + j) grouped
 * by expert ascending, token-ascending inside each expert. */
void ro_bucket(const int32_t* topk_idx, int32_t T, int32_t k, int32_t E,
               int32_t* counts, int32_t* offsets, int32_t* perm_pair);

/* Whole MoE block, src/model.rs:751-818 (+ :820-834 when the shared expert
 * tensors are given, i.e. shared_gate_proj.data != NULL).
 * act_bf16 != 0: x is bf16 bits [T,H]; expert weights are rounded to bf16,
 *   the SwiGLU product h is rounded to bf16 (the GPU's rounding points).
 * act_bf16 == 0: x is float32 [T,H]; everything stays float32.
 * Dot products accumulate in double and round once to float.
 * out is float32 [T,H]. topk_idx/topk_w/counts may be NULL. */
typedef struct ro_moe_weights {
  ro_qtensor gate;          /* mlp.gate.weight            [E, H]    */
  ro_qtensor gate_up_proj;  /* mlp.experts.gate_up_proj   [E, 2I, H] */
  ro_qtensor down_proj;     /* mlp.experts.down_proj      [E, H, I] */
  ro_qtensor shared_gate_proj;   /* [Is, H] (optional) */
  ro_qtensor shared_up_proj;     /* [Is, H] */
  ro_qtensor shared_down_proj;   /* [H, Is] */
  ro_qtensor shared_expert_gate; /* [1, H]  */
  int32_t shared_intermediate;
} ro_moe_weights;

void ro_moe_forward(const ro_moe_weights* w, const void* x, int32_t act_bf16,
                    int32_t T, int32_t H, int32_t I, int32_t E, int32_t k,
                    float* out, int32_t* topk_idx, float* topk_w,
                    int32_t* counts, int32_t n_threads);

/* bf16 helpers (round to nearest even; NaN kept quiet). */
uint16_t ro_f32_to_bf16(float f);
float ro_bf16_to_f32(uint16_t b);

#ifdef __cplusplus
}
#endif
#endif
