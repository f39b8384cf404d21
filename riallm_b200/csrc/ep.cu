// ep.cu -- expert parallelism inside the library: the MoE block with a token
// all-to-all dispatch and combine over NCCL around this rank's expert GEMMs.
//
// No counterpart in the reference: riallm runs every layer on one device
// (src/model.rs:231-258, DeviceSpec::Cuda(usize), src/config.rs:350-372).
// Rank r of W owns experts [r E/W, (r+1) E/W) (contiguous, so the pairs a
// rank sends to r are contiguous in its expert-sorted pair order). A call:
//
//   1. routes this rank's tokens over all E experts (replicated router) and
//      gathers the token rows of its pairs in expert order (x_perm);
//   2. exchanges the per-expert pair counts with every rank (NCCL, grouped
//      point-to-point), then copies the received counts to the host: the
//      one host synchronisation of a call, because NCCL needs the sizes;
//   3. dispatch: one message per peer each way -- rank r gets the rows of
//      its experts (contiguous in the sender's expert order); the rows from
//      all peers land rank-major and one reorder kernel makes them
//      expert-major (peers ascending inside an expert). One message per
//      (peer, expert) instead cost ~3 us of NCCL time per message;
//   4. runs its experts' gate_up / down GEMMs on the received rows;
//   5. return: the float32 output rows are reordered rank-major and sent
//      back one message per peer; they land at the pairs' own positions of
//      the sender's expert-sorted order;
//   6. sums each token's pairs in expert-ascending order with the routing
//      weights (src/model.rs:800-817), as the single-GPU block does.
//
// NCCL is opened at run time (dlopen of libnccl.so.2), so the library has
// no link-time dependency on it; within one process this shares the NCCL
// that torch loaded. Peer memory is touched only by NCCL: no kernel of this
// library reads another GPU's memory, and no load uses TMA multicast.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"

namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    auto sym = [&](const char* n) { return dlsym(h, n); };
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
    api.CommGetAsyncError = reinterpret_cast<decltype(api.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
    api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(sym("ncclGroupStart"));
    api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(sym("ncclGroupEnd"));
    api.Send = reinterpret_cast<decltype(api.Send)>(sym("ncclSend"));
    api.Recv = reinterpret_cast<decltype(api.Recv)>(sym("ncclRecv"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.CommGetAsyncError && api.GroupStart &&
             api.GroupEnd && api.Send && api.Recv && api.GetErrorString;
  });
  return api;
}

int fail(riallm_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}

int nccl_fail(riallm_ctx* ctx, ncclResult_t r, const char* what) {
  return fail(ctx, RIALLM_ERR_CUDA, std::string(what) + ": " + nccl().GetErrorString(r));
}

#define EP_NCCL(ctx, call, what)                        \
  do {                                                  \
    ncclResult_t r_ = (call);                           \
    if (r_ != ncclSuccess) return nccl_fail(ctx, r_, what); \
  } while (0)

#define EP_CUDA(ctx, call, what)                                                               \
  do {                                                                                         \
    cudaError_t e_ = (call);                                                                   \
    if (e_ != cudaSuccess) return fail(ctx, RIALLM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e_)); \
  } while (0)

inline uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

}  // namespace

// Host planning of one exchange (pure function, also exported for tests).
int rl_ep_plan(int world, int e_local, const int32_t* recv_counts, int32_t* expert_counts,
               int32_t* expert_offsets, int32_t* block_pos) {
  if (world <= 0 || e_local <= 0 || !recv_counts || !expert_counts || !expert_offsets || !block_pos)
    return RIALLM_ERR_INVALID;
  int64_t off = 0;
  for (int e = 0; e < e_local; ++e) {
    int64_t tot = 0;
    expert_offsets[e] = (int32_t)off;
    for (int s = 0; s < world; ++s) {
      const int32_t n = recv_counts[s * e_local + e];
      if (n < 0) return RIALLM_ERR_INVALID;
      block_pos[s * e_local + e] = (int32_t)(off + tot);
      tot += n;
    }
    expert_counts[e] = (int32_t)tot;
    off += tot;
    if (off > INT32_MAX) return RIALLM_ERR_CONFIG;
  }
  expert_offsets[e_local] = (int32_t)off;
  return RIALLM_OK;
}

extern "C" {

int32_t riallm_ep_exchange_plan(int32_t world, int32_t e_local, const int32_t* recv_counts,
                                int32_t* expert_counts, int32_t* expert_offsets, int32_t* block_pos) {
  return rl_ep_plan(world, e_local, recv_counts, expert_counts, expert_offsets, block_pos);
}

int32_t riallm_cuda_ep_unique_id(uint8_t* out) {
  if (!out) return RIALLM_ERR_INVALID;
  NcclApi& n = nccl();
  if (!n.ok) return RIALLM_ERR_CONFIG;
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId id;
  if (n.GetUniqueId(&id) != ncclSuccess) return RIALLM_ERR_CUDA;
  memcpy(out, &id, sizeof(id));
  return RIALLM_OK;
}

int32_t riallm_cuda_ep_init(riallm_ctx* ctx, const uint8_t* unique_id, int32_t rank, int32_t world) {
  if (!ctx || !unique_id) return RIALLM_ERR_INVALID;
  if (world < 1 || rank < 0 || rank >= world) return fail(ctx, RIALLM_ERR_CONFIG, "rank outside [0, world)");
  if (ctx->ep_comm) return fail(ctx, RIALLM_ERR_CONFIG, "expert parallelism already initialised on this context");
  NcclApi& n = nccl();
  if (!n.ok) return fail(ctx, RIALLM_ERR_CONFIG, "libnccl.so.2 could not be loaded");
  EP_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  EP_NCCL(ctx, n.CommInitRank(&comm, world, id, rank), "ncclCommInitRank");
  ctx->ep_comm = comm;
  ctx->ep_rank = rank;
  ctx->ep_world = world;
  return RIALLM_OK;
}

int32_t riallm_cuda_ep_destroy(riallm_ctx* ctx) {
  if (!ctx) return RIALLM_ERR_INVALID;
  if (!ctx->ep_comm) return RIALLM_OK;
  cudaSetDevice(ctx->device);
  nccl().CommDestroy(static_cast<ncclComm_t>(ctx->ep_comm));
  ctx->ep_comm = nullptr;
  if (ctx->ep_arena) cudaFree(ctx->ep_arena);
  ctx->ep_arena = nullptr;
  ctx->ep_arena_bytes = 0;
  return RIALLM_OK;
}

int32_t riallm_cuda_ep_async_error(riallm_ctx* ctx) {
  if (!ctx) return RIALLM_ERR_INVALID;
  if (!ctx->ep_comm) return RIALLM_OK;
  ncclResult_t r = ncclSuccess;
  if (nccl().CommGetAsyncError(static_cast<ncclComm_t>(ctx->ep_comm), &r) != ncclSuccess || r != ncclSuccess)
    return fail(ctx, RIALLM_ERR_CUDA, std::string("NCCL asynchronous error: ") + nccl().GetErrorString(r));
  return RIALLM_OK;
}

}  // extern "C"

namespace {

// Moves the rows of W*EL segments between rank-major order (the rows from / to
// each peer back to back, experts ascending inside a peer) and expert-major
// order (the experts' rows back to back, peers ascending inside an expert).
// seg[3i..3i+2] = (rank-major row, expert-major row, rows) of segment i =
// s * EL + e; blockIdx.x is the segment, each warp copies whole rows with
// 16-byte vectors. Row bytes are a multiple of 16 and rows 16-byte aligned.
__global__ void __launch_bounds__(256) ep_segment_copy_kernel(const char* __restrict__ src, char* __restrict__ dst,
                                                              uint64_t row_bytes, const int* __restrict__ seg,
                                                              int to_expert_major) {
  const int rm = seg[3 * blockIdx.x], em = seg[3 * blockIdx.x + 1], cnt = seg[3 * blockIdx.x + 2];
  const int s_off = to_expert_major ? rm : em, d_off = to_expert_major ? em : rm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t nv = row_bytes / 16;
  for (int r = blockIdx.y * 8 + warp; r < cnt; r += gridDim.y * 8) {
    const uint4* sp = reinterpret_cast<const uint4*>(src + (uint64_t)(s_off + r) * row_bytes);
    uint4* dp = reinterpret_cast<uint4*>(dst + (uint64_t)(d_off + r) * row_bytes);
    for (uint64_t v = lane; v < nv; v += 32) dp[v] = __ldcs(sp + v);
  }
}

}  // namespace

int rl_ep_forward(riallm_ctx* ctx, const riallm_moe_weights* w, const void* x, void* out, int T, int H, int I,
                  int E, int k, uint32_t flags, cudaStream_t st, char* base, const rl::MoeLayout& L,
                  uint64_t ep_off) {
  NcclApi& n = nccl();
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->ep_comm);
  const int W = ctx->ep_world, EL = E / W, NS = W * EL;
  const uint64_t rowb = (uint64_t)H * 2, rowy = (uint64_t)H * 4;
  int* rcnt_d = reinterpret_cast<int*>(base + ep_off);
  int* counts = reinterpret_cast<int*>(base + L.counts);
  int* offsets = reinterpret_cast<int*>(base + L.offsets);

  // 2. counts exchange, then the sizes to the host (the call's one host
  // synchronisation: NCCL needs every message size on the host).
  EP_NCCL(ctx, n.GroupStart(), "ncclGroupStart");
  for (int r = 0; r < W; ++r) {
    EP_NCCL(ctx, n.Send(counts + r * EL, EL, ncclInt32, r, comm, st), "ncclSend(counts)");
    EP_NCCL(ctx, n.Recv(rcnt_d + r * EL, EL, ncclInt32, r, comm, st), "ncclRecv(counts)");
  }
  EP_NCCL(ctx, n.GroupEnd(), "ncclGroupEnd");
  std::vector<int32_t>& hbuf = ctx->ep_host;
  hbuf.resize((size_t)NS + E + 1);
  EP_CUDA(ctx, cudaMemcpyAsync(hbuf.data(), rcnt_d, (size_t)NS * 4, cudaMemcpyDeviceToHost, st), "D2H counts");
  EP_CUDA(ctx, cudaMemcpyAsync(hbuf.data() + NS, offsets, (size_t)(E + 1) * 4, cudaMemcpyDeviceToHost, st),
          "D2H offsets");
  EP_CUDA(ctx, cudaStreamSynchronize(st), "cudaStreamSynchronize(exchange sizes)");
  const int32_t* rcnt = hbuf.data();
  const int32_t* off_h = hbuf.data() + NS;

  // Host plan: expert-major counts / offsets / positions, rank-major
  // offsets, and the segment table of the two reorders.
  std::vector<int32_t>& up = ctx->ep_upload;
  up.assign((size_t)2 * EL + 1 + (size_t)3 * NS, 0);
  int32_t* ecnt = up.data();
  int32_t* eoff = ecnt + EL;
  int32_t* seg = eoff + EL + 1;
  std::vector<int32_t> bpos((size_t)NS), rmo((size_t)W + 1, 0);
  if (int rc = rl_ep_plan(W, EL, rcnt, ecnt, eoff, bpos.data())) return fail(ctx, rc, "bad exchange counts");
  const int R = eoff[EL];
  int maxc = 0, maxseg = 0;
  for (int e = 0; e < EL; ++e) maxc = ecnt[e] > maxc ? ecnt[e] : maxc;
  for (int s = 0; s < W; ++s) {
    int64_t o = rmo[s];
    for (int e = 0; e < EL; ++e) {
      const int c = rcnt[s * EL + e];
      seg[3 * (s * EL + e)] = (int32_t)o;
      seg[3 * (s * EL + e) + 1] = bpos[s * EL + e];
      seg[3 * (s * EL + e) + 2] = c;
      maxseg = c > maxseg ? c : maxseg;
      o += c;
    }
    rmo[s + 1] = (int32_t)o;
  }
  if (R > W * T * (k < EL ? k : EL))
    return fail(ctx, RIALLM_ERR_CONFIG, "a rank sent more pairs than T * min(k, experts per rank): every rank must "
                                        "call with the same T");

  // Receive-side arena, sized by R: [upload | xrm | xr | hr | yr | sk_ws];
  // yrm (R rows of float32) reuses xrm + xr, which are dead by then.
  const uint64_t head = align_up((uint64_t)up.size() * 4, 1024);
  const uint64_t xbytes = (uint64_t)R * rowb;
  const uint64_t hbytes = align_up((uint64_t)R * I * 2, 1024);
  const uint64_t ybytes = align_up((uint64_t)R * rowy, 1024);
  const uint64_t skbytes = align_up(rl::tc_sk_ws_bytes(ctx->num_sms, maxc > 0 ? maxc : 1), 1024);
  const uint64_t need = head + align_up(2 * xbytes, 1024) + hbytes + ybytes + skbytes;
  if (need > ctx->ep_arena_bytes) {
    if (ctx->ep_arena) {
      cudaFree(ctx->ep_arena);  // the stream was synchronised above
      ctx->ep_arena = nullptr;
      ctx->ep_arena_bytes = 0;
    }
    const uint64_t bytes = need + need / 4;
    EP_CUDA(ctx, cudaMalloc(&ctx->ep_arena, bytes), "cudaMalloc(expert-parallel receive arena)");
    ctx->ep_arena_bytes = bytes;
  }
  char* eb = static_cast<char*>(ctx->ep_arena);
  int* ecnt_d = reinterpret_cast<int*>(eb);
  int* eoff_d = ecnt_d + EL;
  const int* seg_d = eoff_d + EL + 1;
  char* xrm = eb + head;
  char* xr = xrm + xbytes;
  char* yrm = xrm;
  char* hr = xrm + align_up(2 * xbytes, 1024);
  char* yr = hr + hbytes;
  float* skw = reinterpret_cast<float*>(yr + ybytes);
  EP_CUDA(ctx, cudaMemcpyAsync(eb, up.data(), up.size() * 4, cudaMemcpyHostToDevice, st), "H2D exchange plan");
  const int gy_cap = (8 * ctx->num_sms + NS - 1) / NS;
  const int gy = std::max(1, std::min((maxseg + 7) / 8, gy_cap));

  // 3. dispatch: one message per peer each way. This rank's pairs for rank
  // r's experts are contiguous in its expert-sorted x_perm; the rows from
  // every peer land rank-major and are then reordered expert-major.
  const char* xs = base + L.x_perm;
  {
    rl::PhaseTimer pt(ctx, st, RIALLM_PHASE_DISPATCH);
    EP_NCCL(ctx, n.GroupStart(), "ncclGroupStart");
    for (int r = 0; r < W; ++r) {
      const int c = off_h[(r + 1) * EL] - off_h[r * EL];
      if (c) EP_NCCL(ctx, n.Send(xs + (uint64_t)off_h[r * EL] * rowb, (size_t)c * rowb, ncclUint8, r, comm, st),
                     "ncclSend(tokens)");
    }
    for (int s = 0; s < W; ++s) {
      const int c = rmo[s + 1] - rmo[s];
      if (c) EP_NCCL(ctx, n.Recv(xrm + (uint64_t)rmo[s] * rowb, (size_t)c * rowb, ncclUint8, s, comm, st),
                     "ncclRecv(tokens)");
    }
    EP_NCCL(ctx, n.GroupEnd(), "ncclGroupEnd");
    if (R > 0) {
      ep_segment_copy_kernel<<<dim3(NS, gy), 256, 0, st>>>(xrm, xr, rowb, seg_d, 1);
      EP_CUDA(ctx, cudaGetLastError(), "expert-major reorder");
      ctx->launches += 1;
    }
  }

  // 4. this rank's experts on the received rows.
  if (R > 0) {
    rl::TcGemmArgs g{};
    g.w = w->gate_up_proj;
    g.K = H;
    g.rows_per_expert = 2 * I;
    g.a1_offset = I;
    g.m_step = 128;
    g.m_tiles = I / 128;
    g.b = xr;
    g.P = R;
    g.counts = ecnt_d;
    g.offsets = eoff_d;
    g.E = EL;
    g.swiglu = true;
    g.h_pair_perm = w->down_proj.qtype == RIALLM_COMPRESSION_FOUR_BIT;
    g.h_out = reinterpret_cast<uint16_t*>(hr);
    g.ld_out = I;
    g.status = ctx->d_status;
    g.max_pairs_per_expert = maxc;
    g.sk_ws = skw;
    g.sk_flags = reinterpret_cast<int*>(base + L.sync + rl::kSkFlagsOffset);
    g.pdl = false;  // follows the reorder; its counts come from the plan upload
    g.flag_wait_ns = ctx->flag_wait_ns;
    rl::TcGemmArgs d = g;
    d.w = w->down_proj;
    d.K = I;
    d.rows_per_expert = H;
    d.a1_offset = 128;
    d.m_step = 256;
    d.m_tiles = H / 256;
    d.b = hr;
    d.swiglu = false;
    d.h_pair_perm = false;
    d.h_out = nullptr;
    d.y_out = reinterpret_cast<float*>(yr);
    d.ld_out = H;
    d.pdl = true;
    g.next = &d;
    {
      rl::PhaseTimer pt(ctx, st, RIALLM_PHASE_GATE_UP);
      EP_CUDA(ctx, rl::launch_tc_gemm(g, ctx->num_sms, st), "expert gate_up (tcgen05)");
      ctx->launches += 1;
    }
    {
      rl::PhaseTimer pt(ctx, st, RIALLM_PHASE_DOWN);
      EP_CUDA(ctx, rl::launch_tc_gemm(d, ctx->num_sms, st), "expert down (tcgen05)");
      ctx->launches += 1;
    }
  }

  // 5. return: the output rows reordered rank-major, one message per peer
  // each way; the rows from rank r land at r's experts' positions of this
  // rank's expert-sorted y_perm, which are contiguous and in the order the
  // dispatch sent them.
  float* y_perm = reinterpret_cast<float*>(base + L.y_perm);
  {
    rl::PhaseTimer pt(ctx, st, RIALLM_PHASE_RETURN);
    if (R > 0) {
      ep_segment_copy_kernel<<<dim3(NS, gy), 256, 0, st>>>(yr, yrm, rowy, seg_d, 0);
      EP_CUDA(ctx, cudaGetLastError(), "rank-major reorder");
      ctx->launches += 1;
    }
    EP_NCCL(ctx, n.GroupStart(), "ncclGroupStart");
    for (int s = 0; s < W; ++s) {
      const int c = rmo[s + 1] - rmo[s];
      if (c) EP_NCCL(ctx, n.Send(yrm + (uint64_t)rmo[s] * rowy, (size_t)c * rowy, ncclUint8, s, comm, st),
                     "ncclSend(outputs)");
    }
    for (int r = 0; r < W; ++r) {
      const int c = off_h[(r + 1) * EL] - off_h[r * EL];
      if (c) EP_NCCL(ctx, n.Recv(reinterpret_cast<char*>(y_perm) + (uint64_t)off_h[r * EL] * rowy, (size_t)c * rowy,
                                 ncclUint8, r, comm, st),
                     "ncclRecv(outputs)");
    }
    EP_NCCL(ctx, n.GroupEnd(), "ncclGroupEnd");
  }
  (void)x;
  // 6. the weighted sum per token, expert-ascending (all E experts).
  {
    rl::PhaseTimer pt(ctx, st, RIALLM_PHASE_COMBINE);
    EP_CUDA(ctx, rl::launch_combine(y_perm, reinterpret_cast<const int*>(base + L.inv_pos),
                                    reinterpret_cast<const int*>(base + L.topk_idx),
                                    reinterpret_cast<const float*>(base + L.topk_w), T, k, H, nullptr, nullptr, out,
                                    true, (flags & RIALLM_MOE_ADD_TO_OUT) != 0, st, 0, 1 << 30, true),
            "combine");
    ctx->launches += 1;
  }
  return RIALLM_OK;
}

// Bytes after the regular layout that rl_ep_forward needs there (the
// received counts); everything sized by the received rows lives in the
// context's expert-parallel arena.
uint64_t rl_ep_extra_bytes(int T, int H, int I, int E, int k, int W, int num_sms) {
  (void)T, (void)H, (void)I, (void)k, (void)num_sms;
  return align_up((uint64_t)W * (E / W) * 4, 1024) + 1024;
}
