// internal.h -- declarations shared by the translation units of
// libriallm_cuda. Not part of the public ABI (include/riallm_cuda.h is).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "riallm_cuda.h"

struct riallm_ctx {
  int device = 0;
  int num_sms = 148;
  std::string last_error;
  // Scratch arena for one MoE block call: grown with cudaMalloc on demand,
  // never shrunk, freed with the context.
  void* arena = nullptr;
  uint64_t arena_bytes = 0;
  // Arenas outgrown by a larger call. They stay allocated until the context
  // is destroyed: a CUDA graph that captured an earlier call still uses its
  // arena's address when it is replayed.
  std::vector<void*> retired_arenas;
  // Device status word written by kernels whose bounded waits expired.
  int* d_status = nullptr;
  // Split-key attention workspace (rl::attn_ws_bytes), allocated with the
  // context so that graph-captured attention calls never see it move.
  void* attn_ws = nullptr;
  // Kernel launches issued by this context.
  uint64_t launches = 0;
  // Phase profiling: event pairs recorded per call, summed on read.
  bool profiling = false;
  struct PhaseEvents {
    int phase;
    cudaEvent_t start, stop;
  };
  std::vector<PhaseEvents> pending;
  std::vector<cudaEvent_t> event_pool;
  uint64_t profiled_calls = 0;
  // Bound (ns) of a kernel's wait for work published by other CTAs of the
  // same launch (riallm_cuda_ctx_set_wait_limit; 0 = the default 1 s), and
  // the test hook that makes the next MoE call's such wait expire.
  uint64_t flag_wait_ns = 0;
  bool expire_next_wait = false;
  // Expert parallelism (riallm_cuda_ep_init): the NCCL communicator of this
  // context's rank, host staging of one call's exchange sizes, and the
  // receive-side arena (sized by the rows a call actually receives; grown,
  // never shrunk, freed with the communicator).
  void* ep_comm = nullptr;
  int ep_rank = 0, ep_world = 1;
  std::vector<int32_t> ep_host, ep_upload;
  void* ep_arena = nullptr;
  uint64_t ep_arena_bytes = 0;
  // Peer-memory transport (riallm_cuda_ep_peer_init): the shape it was set
  // up for, this rank's symmetric buffer (same layout on every rank, mapped
  // by the peers through CUDA IPC), the peers' mapped bases, and this
  // rank's local buffers (plan, epoch, counters, expert intermediates).
  bool ep_peer = false;
  int ep_peer_T = 0, ep_peer_H = 0, ep_peer_I = 0, ep_peer_E = 0, ep_peer_k = 0;
  void* ep_sym = nullptr;
  std::vector<void*> ep_peer_open;
  void* ep_peer_local = nullptr;
};

namespace rl {

// Phase profiling (riallm_cuda_profile_enable): an event pair around a
// phase on the call's stream, recorded only while profiling is on.
inline cudaEvent_t take_event(riallm_ctx* ctx) {
  if (!ctx->event_pool.empty()) {
    cudaEvent_t e = ctx->event_pool.back();
    ctx->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}
struct PhaseTimer {
  riallm_ctx* ctx;
  cudaStream_t st;
  int phase;
  cudaEvent_t start = nullptr;
  PhaseTimer(riallm_ctx* c, cudaStream_t s, int p) : ctx(c), st(s), phase(p) {
    if (ctx->profiling && (start = take_event(ctx))) cudaEventRecord(start, st);
  }
  ~PhaseTimer() {
    if (!start) return;
    cudaEvent_t stop = take_event(ctx);
    if (!stop) {
      ctx->event_pool.push_back(start);
      return;
    }
    cudaEventRecord(stop, st);
    ctx->pending.push_back({phase, start, stop});
  }
};

// Split-key attention: when the (sequence, kv head, token) groups of a call
// fill fewer than 2 CTAs per SM, each group's keys are split over several
// CTAs (at most 4 per SM in total) whose partial softmax sums are merged by
// the group's last CTA. The workspace holds one completion counter per group
// (zero between calls) and the partials: per CTA, REP maxima, REP sums and
// REP x D accumulators (REP <= 8, D <= 128).
constexpr int kAttnMaxRep = 8, kAttnMaxD = 128;
constexpr uint64_t kAttnCounterBytes = 4096;
inline uint64_t attn_ws_bytes(int num_sms) {
  return kAttnCounterBytes + (uint64_t)4 * num_sms * kAttnMaxRep * (kAttnMaxD + 2) * sizeof(float);
}

// Offsets of the MoE scratch buffers inside one arena (all 1 KiB aligned).
// The first kSyncBytes of a layout hold counters that must read zero
// between calls: the router's completion counter at offset 0 and the
// expert GEMM's split-tile counters (one per SM) from kSkFlagsOffset.
constexpr uint64_t kSyncBytes = 4096;
constexpr uint64_t kSkFlagsOffset = 256;
struct MoeLayout {
  uint64_t sync, sk_ws, topk_idx, topk_w, counts, offsets, perm_pair, inv_pos;
  uint64_t x_perm, h_perm, y_perm, proj;
  uint64_t cta_base;  // router per-CTA pair bases (multi-CTA sort)
  // Token-tiled router calls: the quantized router weight decoded once to
  // float32 [E, H] (0 bytes when the router keeps one token per CTA).
  uint64_t gate_f32, gate_f32_bytes;
  uint64_t sh_g, sh_u, sh_h, sh_y, sh_gate;
  uint64_t total;
};
// with_sk: reserve the expert GEMM's split-tile workspace (bf16 only).
MoeLayout moe_layout(int T, int H, int I, int E, int k, int act_dtype, int shared_I, int num_sms,
                     bool with_sk = true);

cudaError_t launch_dequant(const riallm_qtensor& t, int mode, void* dst, int dst_dtype,
                           int num_sms, cudaStream_t stream);
cudaError_t launch_quantize(int qtype, const float* src, uint64_t n, uint8_t* data,
                            float* scales, float* zeros, int num_sms, cudaStream_t stream);

// Router (fixed-order fp32 dot products, own exp, stable top-k) fused with
// the counting sort of the T*k (token, choice) pairs by expert.
constexpr int kRouterThreads = 256;
struct RouterArgs {
  const void* x;
  int x_bf16;
  const void* gdata;  // router weight [E, H]: float32, NF4 or 8-bit codes
  const float* gscales;
  const float* gzeros;
  uint64_t n_scales, n_zeros;
  int T, H, E, k;
  int* topk_idx;
  float* topk_w;
  int* counts;
  int* offsets;
  int* perm_pair;
  int* inv_pos;
  unsigned* done;  // zero between calls; the last CTA resets it
  // Calls of more than kSortOneCta pairs: per group of kSortGroup tokens
  // and expert, the group's pair count (zeroed before the router runs),
  // then the base of its pairs (router_cta_bytes()).
  int* cta_base;
  // float32 router weight whose base is 32-byte aligned: each lane reads its
  // 8-float chunk with one 256-bit load (a warp reads 1 KiB contiguously).
  int gate_v8;
};
// Pairs (T * k) up to which the router's last CTA sorts all pairs by itself;
// larger calls sort with every router CTA and a scatter kernel.
constexpr int64_t kSortOneCta = 16384;
constexpr int kMaxExperts = 256;
// Tokens per router CTA (1 for decode-sized calls).
int router_tile_tokens(int T, int H);
constexpr int kSortGroup = 64;  // tokens per group of the multi-CTA sort (a multiple of every tile)
inline uint64_t router_cta_bytes(int T, int H, int E) {
  (void)H;
  return (uint64_t)((T + kSortGroup - 1) / kSortGroup) * E * 4;
}
cudaError_t launch_router(const RouterArgs& a, int gate_qtype, cudaStream_t stream);
// Gathers token rows into expert-sorted pair order. pair_perm (bf16 only)
// stores each group of 8 columns in the K order of the NF4 tensor-core
// decode: [0,4,1,5,2,6,3,7].
// row_begin / row_end (device ints, optional): only rows [*row_begin,
// *row_end) are written (an expert-parallel rank's experts).
cudaError_t launch_gather(const void* x, bool x_bf16, const int* perm_pair, int k, int P, int H,
                          void* x_perm, bool pair_perm, cudaStream_t stream,
                          const int* row_begin = nullptr, const int* row_end = nullptr);
// out[t] = sum over t's pairs in expert-ascending order of w * y_perm[pos]
// (+ shared expert), optional residual add, cast to the activation dtype.
// Pairs whose expert lies outside [e_begin, e_end) are skipped. round_w:
// the routing weights are rounded to bf16 first (bf16 activations,
// src/model.rs:800-802).
cudaError_t launch_combine(const float* y_perm, const int* inv_pos, const int* topk_idx,
                           const float* topk_w, int T, int k, int H, const float* shared_y,
                           const float* shared_gate, void* out, bool out_bf16, bool add_to_out,
                           cudaStream_t stream, int e_begin, int e_end, bool round_w);

// Generic CUDA-core grouped GEMM with on-the-fly dequant (float32 path and
// the shared expert): Y[pos, r] = sum_c X[pos, c] * W[row_base(e) + r, c].
// X is float32 or bf16 [P, K]; Y float32 [P, ldy].
struct GroupedF32Args {
  riallm_qtensor w;
  int K;
  int rows;             // output rows per expert
  int rows_per_expert;  // row stride between experts inside w
  int row_offset;       // first weight row used inside an expert
  const void* x;
  bool x_bf16;
  float* y;
  int ldy;
  int y_col0;
  const int* counts;   // nullptr: a single group of P rows
  const int* offsets;
  int E;
  int P;
  bool round_w_bf16;
};
cudaError_t launch_grouped_f32(const GroupedF32Args& a, cudaStream_t stream);
// h[pos, i] = silu(g[pos, i]) * u[pos, i] (optionally rounded to bf16).
cudaError_t launch_swiglu(const float* g, int ldg, const float* u, int ldu, void* h, int ldh,
                          int P, int I, bool h_bf16, cudaStream_t stream);

// tcgen05 grouped expert GEMM with in-register dequant (bf16 activations).
struct TcGemmArgs {
  riallm_qtensor w;
  int K;                // reduction length (H for gate_up, I for down)
  int rows_per_expert;  // 2I (gate_up) or H (down)
  int a1_offset;        // row offset of operand 1 inside a tile: I or 128
  int m_step;           // rows per M tile step: 128 (gate_up) or 256 (down)
  int m_tiles;          // I/128 or H/256
  const void* b;        // bf16 [P, K] in pair order (x_perm or h_perm)
  int P;
  const int* counts;
  const int* offsets;
  int E;
  bool swiglu;          // gate_up epilogue (h = silu(D0) * D1) vs down (y = D0 | D1)
  bool h_pair_perm;     // store h in the NF4 decode's K order (the down weights are NF4)
  uint16_t* h_out;      // [P, ld_out] bf16 when swiglu
  float* y_out;         // [P, ld_out] f32 otherwise
  int ld_out;
  int* status;
  int max_pairs_per_expert;  // upper bound on any expert's pair count (<= T)
  float* sk_ws;              // split-tile partial sums, tc_sk_ws_bytes(); null: whole tiles per CTA
  int* sk_flags;             // num_sms counters, zero between launches
  // Launch with programmatic stream serialization: the prologue and the
  // weight stream may start while the previous kernel (which must not
  // produce the routing counts) is still running; token tiles, outputs and
  // the split-tile workspace are touched only after griddepcontrol.wait.
  bool pdl;
  // The expert GEMM launched right after this one on the same stream (the
  // down projection after gate_up), or null. When its weights have this
  // launch's format and tiles are decode-sized (<= 64 pairs per expert),
  // each CTA, once it has issued its last weight loads,
  // prefetches into L2 the first weight stages that the same CTA index
  // reads in the next launch.
  const TcGemmArgs* next = nullptr;
  // Bound of the split-tile owner's wait for partial sums (0: the default,
  // kWaitLimitNs) and a count added to the awaited value (test hook).
  uint64_t flag_wait_ns = 0;
  int flag_extra = 0;
};
// Bytes of the split-tile workspace of launch_tc_gemm: one slot of
// 2 operands x 128 rows x (64 or 128) f32 columns per CTA (= per SM).
inline uint64_t tc_sk_ws_bytes(int num_sms, int max_pairs_per_expert) {
  return (uint64_t)num_sms * 2u * 128u * (max_pairs_per_expert <= 64 ? 64u : 128u) * 4u;
}
cudaError_t launch_tc_gemm(const TcGemmArgs& a, int num_sms, cudaStream_t stream);

// Driver entry point for cuTensorMapEncodeTiled (resolved at run time).
CUresult encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                              uint64_t dim0, uint64_t dim1, uint64_t row_stride_bytes,
                              uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle);

}  // namespace rl

// Expert-parallel block with the token all-to-all (ep.cu): the receive-side
// scratch that follows a call's regular layout, and the call's exchange,
// expert GEMMs and combine after routing and gathering (ep_off = where the
// receive side starts in the arena).
uint64_t rl_ep_extra_bytes(int T, int H, int I, int E, int k, int W, int num_sms);
int rl_ep_forward(riallm_ctx* ctx, const riallm_moe_weights* w, const void* x, void* out, int T, int H, int I,
                  int E, int k, uint32_t flags, cudaStream_t st, char* base, const rl::MoeLayout& L,
                  uint64_t ep_off);
int rl_ep_plan(int world, int e_local, const int32_t* recv_counts, int32_t* expert_counts,
               int32_t* expert_offsets, int32_t* block_pos);
// The same block over the peer-memory transport (riallm_cuda_ep_peer_init):
// no host synchronisation; combine reads the returned rows from the
// symmetric buffer.
int rl_ep_peer_forward(riallm_ctx* ctx, const riallm_moe_weights* w, void* out, int T, int H, int I, int E, int k,
                       uint32_t flags, cudaStream_t st, char* base, const rl::MoeLayout& L);
