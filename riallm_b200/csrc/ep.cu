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

#include "common.cuh"
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
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
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
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(sym("ncclAllGather"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.CommGetAsyncError && api.GroupStart &&
             api.GroupEnd && api.Send && api.Recv && api.AllGather && api.GetErrorString;
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

// Frees the peer transport of a context (defined with the transport below).
static void peer_teardown_ctx(riallm_ctx* ctx);

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
  peer_teardown_ctx(ctx);
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

// ===================================================== peer-memory transport
//
// The same exchange without NCCL on the data path and without a host
// synchronisation, so a call can be captured in a CUDA graph. Every rank
// owns a symmetric buffer (the same layout on every rank) that its peers map
// through CUDA IPC: four arrays of W epoch flags and the receive areas for
// token rows (expert-major) and for returned output rows (this rank's
// expert-sorted pair order). A call:
//
//   1. all-gathers the W x E pair-count matrix (NCCL, on the stream);
//   2. plan kernel: bumps the call's epoch n, derives from the matrix where
//      each of this rank's rows lands at its owner and where each received
//      row goes back, then waits until every receiver has consumed this
//      rank's rows of call n-1 (free_x);
//   3. dispatch kernel: copies each pair row straight into its owner's
//      receive area with stores over NVLink; the CTA that finishes last
//      publishes arrived_x = n at every peer (release, system scope);
//   4. waits for arrived_x = n from every peer, runs the expert GEMMs,
//      tells every sender its rows were consumed (free_x = n);
//   5. waits until every home rank has consumed call n-1's returns (free_y),
//      copies each output row into its home rank's return area at the
//      pair's own position, publishes arrived_y = n;
//   6. waits for arrived_y = n from every peer, combines, publishes
//      free_y = n.
//
// Every wait is bounded (RIALLM_ERR_TIMEOUT in the context's status word);
// every peer address is bounds-checked against the receive areas before it
// is stored to. Stores are plain st.global to mapped peer memory: no TMA,
// no multicast.
namespace {

constexpr int kArrX = 0, kArrY = 1, kFreeX = 2, kFreeY = 3;
constexpr uint64_t kPeerWaitNs = 5000ull * 1000ull * 1000ull;  // 5 s

struct PeerLayout {
  int cap_x, cap_y, maxp;
  // symmetric buffer
  uint64_t flags, xr, ret, total;
  // local buffer
  uint64_t epoch, done, cmat, dest_base, ecnt, eoff, rcv_pos, ret_base, peers, hr, yr, skw, ltotal;
};

PeerLayout peer_layout(int W, int T, int H, int I, int E, int k, int num_sms) {
  PeerLayout p{};
  const int EL = E / W;
  p.cap_x = W * T * (k < EL ? k : EL);  // rows this rank can receive
  p.cap_y = T * k;                      // this rank's own pairs
  p.maxp = W * T < p.cap_x ? W * T : p.cap_x;  // an expert gets at most one pair per token
  uint64_t o = 0;
  auto take = [&](uint64_t b) {
    const uint64_t r = o;
    o = align_up(o + b, 1024);
    return r;
  };
  p.flags = take(4ull * W * 8);
  p.xr = take((uint64_t)p.cap_x * H * 2);
  p.ret = take((uint64_t)p.cap_y * H * 4);
  p.total = o;
  o = 0;
  p.epoch = take(8);
  p.done = take(16);
  p.cmat = take((uint64_t)W * E * 4);
  p.dest_base = take((uint64_t)E * 4);
  p.ecnt = take((uint64_t)EL * 4);
  p.eoff = take((uint64_t)(EL + 1) * 4);
  p.rcv_pos = take((uint64_t)W * EL * 4);
  p.ret_base = take((uint64_t)W * EL * 4);
  p.peers = take((uint64_t)W * 8);
  p.hr = take((uint64_t)p.cap_x * I * 2);
  p.yr = take((uint64_t)p.cap_x * H * 4);
  p.skw = take(rl::tc_sk_ws_bytes(num_sms, p.maxp));
  p.ltotal = o;
  return p;
}

__device__ __forceinline__ uint64_t* flag_at(char* sym_base, int which, int W, int from) {
  return reinterpret_cast<uint64_t*>(sym_base) + which * W + from;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0: waits, at most limit_ns, until flags[0..W) >= target; records
// RIALLM_ERR_TIMEOUT otherwise.
__device__ void wait_peer_flags(const uint64_t* flags, int W, uint64_t target, uint64_t limit_ns, int* status) {
  const uint64_t t0 = rl::globaltimer_ns();
  for (;;) {
    bool ok = true;
    for (int s = 0; s < W && ok; ++s) ok = ld_acquire_sys(flags + s) >= target;
    if (ok) return;
    if (rl::globaltimer_ns() - t0 > limit_ns) {
      atomicExch(status, RIALLM_ERR_TIMEOUT);
      return;
    }
    __nanosleep(200);
  }
}

struct PeerArgs {
  char* const* peers;  // [W] symmetric bases, this rank's own at [me]
  char* sym;           // this rank's symmetric base
  char* loc;           // this rank's local buffer
  int* status;
  uint64_t wait_ns;
  int W, me, E, EL;
  PeerLayout L;
};

// Step 2 (one thread): epoch, plan, then wait for free_x >= n - 1.
__global__ void ep_peer_plan_kernel(PeerArgs a) {
  if (threadIdx.x != 0) return;
  uint64_t* epoch = reinterpret_cast<uint64_t*>(a.loc + a.L.epoch);
  const uint64_t n = *epoch + 1;
  *epoch = n;
  const int W = a.W, E = a.E, EL = a.EL, me = a.me;
  const int* C = reinterpret_cast<const int*>(a.loc + a.L.cmat);  // C[s * E + e]: rank s's pairs of expert e
  int* dest_base = reinterpret_cast<int*>(a.loc + a.L.dest_base);
  int* ecnt = reinterpret_cast<int*>(a.loc + a.L.ecnt);
  int* eoff = reinterpret_cast<int*>(a.loc + a.L.eoff);
  int* rcv_pos = reinterpret_cast<int*>(a.loc + a.L.rcv_pos);
  int* ret_base = reinterpret_cast<int*>(a.loc + a.L.ret_base);
  // This rank's receive area: its experts in order, ranks ascending inside
  // an expert.
  int off = 0;
  for (int el = 0; el < EL; ++el) {
    const int e = me * EL + el;
    eoff[el] = off;
    int c = 0;
    for (int s = 0; s < W; ++s) {
      rcv_pos[s * EL + el] = off + c;
      c += C[s * E + e];
    }
    ecnt[el] = c;
    off += c;
  }
  eoff[EL] = off;
  // Where this rank's rows of expert e start in the owner's receive area.
  for (int r = 0; r < W; ++r) {
    int o = 0;
    for (int el = 0; el < EL; ++el) {
      const int e = r * EL + el;
      int before = 0;
      for (int s = 0; s < me; ++s) before += C[s * E + e];
      dest_base[e] = o + before;
      for (int s = 0; s < W; ++s) o += C[s * E + e];
    }
  }
  // Where rank s's pairs of this rank's expert e sit in s's expert-sorted
  // order (s's router offsets: the prefix of its counts).
  for (int s = 0; s < W; ++s) {
    int o = 0;
    for (int e = 0; e < E; ++e) {
      if (e / EL == me) ret_base[s * EL + (e - me * EL)] = o;
      o += C[s * E + e];
    }
  }
  wait_peer_flags(flag_at(a.sym, kFreeX, W, 0), W, n - 1, a.wait_ns, a.status);
}

// Thread 0: wait until flags[which][0..W) of this rank >= epoch - back.
__global__ void ep_peer_wait_kernel(PeerArgs a, int which, int back) {
  if (threadIdx.x != 0) return;
  const uint64_t n = *reinterpret_cast<const uint64_t*>(a.loc + a.L.epoch);
  wait_peer_flags(flag_at(a.sym, which, a.W, 0), a.W, n - back, a.wait_ns, a.status);
}

// Lane s < W: flags[which][me] of rank s = epoch.
__global__ void ep_peer_signal_kernel(PeerArgs a, int which) {
  const int s = threadIdx.x;
  if (s >= a.W) return;
  const uint64_t n = *reinterpret_cast<const uint64_t*>(a.loc + a.L.epoch);
  __threadfence_system();
  st_release_sys(flag_at(a.peers[s], which, a.W, a.me), n);
}

// The last CTA to finish (a local counter it resets) publishes `which` = n at
// every peer, after every CTA's stores were fenced at system scope.
__device__ void publish_when_done(const PeerArgs& a, int counter, int which) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* done = reinterpret_cast<unsigned*>(a.loc + a.L.done) + counter;
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      __threadfence_system();
      const uint64_t n = *reinterpret_cast<const uint64_t*>(a.loc + a.L.epoch);
      for (int s = 0; s < a.W; ++s) st_release_sys(flag_at(a.peers[s], which, a.W, a.me), n);
      *done = 0;
    }
  }
}

// Copies `row_bytes` (a multiple of 16) from src to dst, one warp.
__device__ __forceinline__ void warp_copy_row(const char* __restrict__ src, char* dst, uint64_t row_bytes,
                                              int lane) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  const int n16 = (int)(row_bytes / 16);
  for (int i0 = lane; i0 < n16; i0 += 32 * 8) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (i0 + 32 * u < n16) v[u] = __ldcs(s + i0 + 32 * u);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (i0 + 32 * u < n16) d[i0 + 32 * u] = v[u];
  }
}

// Step 3: pair row i of x_perm (expert e = the one whose offsets range holds
// i) to its owner's receive area.
__global__ void __launch_bounds__(256) ep_peer_dispatch_kernel(PeerArgs a, const char* __restrict__ x_perm,
                                                               const int* __restrict__ offsets, int P,
                                                               uint64_t rowb) {
  const int lane = threadIdx.x & 31;
  const int* dest_base = reinterpret_cast<const int*>(a.loc + a.L.dest_base);
  for (int i = blockIdx.x * 8 + (threadIdx.x >> 5); i < P; i += gridDim.x * 8) {
    int lo = 0, hi = a.E;  // largest e with offsets[e] <= i
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(offsets + mid) <= i) lo = mid;
      else hi = mid;
    }
    const int e = lo, r = e / a.EL;
    const int row = dest_base[e] + (i - __ldg(offsets + e));
    if (row < 0 || row >= a.L.cap_x || r >= a.W) {
      if (lane == 0) atomicExch(a.status, RIALLM_ERR_INVALID);
      continue;
    }
    warp_copy_row(x_perm + (uint64_t)i * rowb, a.peers[r] + a.L.xr + (uint64_t)row * rowb, rowb, lane);
  }
  publish_when_done(a, 0, kArrX);
}

// Step 5: received row q (expert el, from rank s, its j-th pair of that
// expert) back to position ret_base[s][el] + j of rank s's return area.
__global__ void __launch_bounds__(256) ep_peer_return_kernel(PeerArgs a, uint64_t rowy) {
  const int lane = threadIdx.x & 31;
  const int* C = reinterpret_cast<const int*>(a.loc + a.L.cmat);
  const int* eoff = reinterpret_cast<const int*>(a.loc + a.L.eoff);
  const int* rcv_pos = reinterpret_cast<const int*>(a.loc + a.L.rcv_pos);
  const int* ret_base = reinterpret_cast<const int*>(a.loc + a.L.ret_base);
  const char* yr = a.loc + a.L.yr;
  const int R = eoff[a.EL];
  for (int q = blockIdx.x * 8 + (threadIdx.x >> 5); q < R; q += gridDim.x * 8) {
    int el = 0, hi = a.EL;  // largest el with eoff[el] <= q
    while (hi - el > 1) {
      const int mid = (el + hi) >> 1;
      if (eoff[mid] <= q) el = mid;
      else hi = mid;
    }
    const int e = a.me * a.EL + el;
    int s = 0;
    while (s + 1 < a.W && q >= rcv_pos[s * a.EL + el] + C[s * a.E + e]) ++s;
    const int pos = ret_base[s * a.EL + el] + (q - rcv_pos[s * a.EL + el]);
    if (pos < 0 || pos >= a.L.cap_y || q >= a.L.cap_x) {
      if (lane == 0) atomicExch(a.status, RIALLM_ERR_INVALID);
      continue;
    }
    warp_copy_row(yr + (uint64_t)q * rowy, a.peers[s] + a.L.ret + (uint64_t)pos * rowy, rowy, lane);
  }
  publish_when_done(a, 1, kArrY);
}

}  // namespace

namespace {

void peer_teardown(riallm_ctx* ctx) {
  if (!ctx->ep_peer && !ctx->ep_sym && !ctx->ep_peer_local) return;
  cudaSetDevice(ctx->device);
  cudaDeviceSynchronize();
  for (void* p : ctx->ep_peer_open)
    if (p) cudaIpcCloseMemHandle(p);
  ctx->ep_peer_open.clear();
  if (ctx->ep_sym) cudaFree(ctx->ep_sym);
  if (ctx->ep_peer_local) cudaFree(ctx->ep_peer_local);
  ctx->ep_sym = nullptr;
  ctx->ep_peer_local = nullptr;
  ctx->ep_peer = false;
}

}  // namespace

extern "C" {

int32_t riallm_cuda_ep_peer_init(riallm_ctx* ctx, int32_t max_tokens, int32_t H, int32_t I, int32_t E, int32_t k) {
  if (!ctx) return RIALLM_ERR_INVALID;
  if (!ctx->ep_comm) return fail(ctx, RIALLM_ERR_CONFIG, "riallm_cuda_ep_init was not called on this context");
  const int W = ctx->ep_world, me = ctx->ep_rank;
  if (max_tokens < 1 || H <= 0 || I <= 0 || E <= 0 || k <= 0 || k > E || E > 256 || k > 16 || E % W || H % 256 ||
      I % 256)
    return fail(ctx, RIALLM_ERR_CONFIG, "peer transport: need T >= 1, H and I multiples of 256, k <= E <= 256, "
                                        "k <= 16 and E a multiple of the world size");
  NcclApi& n = nccl();
  EP_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  peer_teardown(ctx);
  const PeerLayout L = peer_layout(W, max_tokens, H, I, E, k, ctx->num_sms);
  auto bail = [&](int code, const std::string& msg) {
    peer_teardown(ctx);
    return fail(ctx, code, msg);
  };
  if (cudaMalloc(&ctx->ep_sym, L.total) != cudaSuccess || cudaMalloc(&ctx->ep_peer_local, L.ltotal) != cudaSuccess)
    return bail(RIALLM_ERR_CUDA, "cudaMalloc(peer transport buffers)");
  if (cudaMemset(ctx->ep_sym, 0, L.xr) != cudaSuccess ||
      cudaMemset(ctx->ep_peer_local, 0, L.cmat) != cudaSuccess)
    return bail(RIALLM_ERR_CUDA, "cudaMemset(peer transport flags)");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ctx->ep_sym) != cudaSuccess) return bail(RIALLM_ERR_CUDA, "cudaIpcGetMemHandle");
  // Every rank's flags are zero before any rank can learn its handle.
  if (cudaDeviceSynchronize() != cudaSuccess) return bail(RIALLM_ERR_CUDA, "cudaDeviceSynchronize");
  char* dh = nullptr;
  cudaStream_t st = nullptr;
  std::vector<cudaIpcMemHandle_t> hs(W);
  if (cudaMalloc(&dh, (size_t)W * sizeof(h)) != cudaSuccess || cudaStreamCreate(&st) != cudaSuccess ||
      cudaMemcpy(dh + (size_t)me * sizeof(h), &h, sizeof(h), cudaMemcpyHostToDevice) != cudaSuccess) {
    if (dh) cudaFree(dh);
    if (st) cudaStreamDestroy(st);
    return bail(RIALLM_ERR_CUDA, "peer handle exchange buffers");
  }
  const ncclResult_t r = n.AllGather(dh + (size_t)me * sizeof(h), dh, sizeof(h), ncclUint8,
                                     static_cast<ncclComm_t>(ctx->ep_comm), st);
  const bool ok = r == ncclSuccess && cudaStreamSynchronize(st) == cudaSuccess &&
                  cudaMemcpy(hs.data(), dh, (size_t)W * sizeof(h), cudaMemcpyDeviceToHost) == cudaSuccess;
  cudaFree(dh);
  cudaStreamDestroy(st);
  if (!ok) return bail(RIALLM_ERR_CUDA, "peer handle exchange (ncclAllGather)");
  std::vector<char*> bases(W, nullptr);
  ctx->ep_peer_open.assign(W, nullptr);
  for (int s = 0; s < W; ++s) {
    if (s == me) {
      bases[s] = static_cast<char*>(ctx->ep_sym);
      continue;
    }
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, hs[s], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
      return bail(RIALLM_ERR_CUDA, "cudaIpcOpenMemHandle (peer " + std::to_string(s) + ")");
    ctx->ep_peer_open[s] = p;
    bases[s] = static_cast<char*>(p);
  }
  if (cudaMemcpy(static_cast<char*>(ctx->ep_peer_local) + L.peers, bases.data(), (size_t)W * sizeof(char*),
                 cudaMemcpyHostToDevice) != cudaSuccess)
    return bail(RIALLM_ERR_CUDA, "peer base upload");
  ctx->ep_peer = true;
  ctx->ep_peer_T = max_tokens;
  ctx->ep_peer_H = H;
  ctx->ep_peer_I = I;
  ctx->ep_peer_E = E;
  ctx->ep_peer_k = k;
  return RIALLM_OK;
}

}  // extern "C"

int rl_ep_peer_forward(riallm_ctx* ctx, const riallm_moe_weights* w, void* out, int T, int H, int I, int E, int k,
                       uint32_t flags, cudaStream_t st, char* base, const rl::MoeLayout& L) {
  NcclApi& n = nccl();
  const int W = ctx->ep_world, EL = E / W, P = T * k;
  const PeerLayout pl = peer_layout(W, ctx->ep_peer_T, H, I, E, k, ctx->num_sms);
  char* sym = static_cast<char*>(ctx->ep_sym);
  char* loc = static_cast<char*>(ctx->ep_peer_local);
  PeerArgs a{};
  a.peers = reinterpret_cast<char* const*>(loc + pl.peers);
  a.sym = sym;
  a.loc = loc;
  a.status = ctx->d_status;
  a.wait_ns = ctx->flag_wait_ns ? ctx->flag_wait_ns : kPeerWaitNs;
  a.W = W;
  a.me = ctx->ep_rank;
  a.E = E;
  a.EL = EL;
  a.L = pl;
  const uint64_t rowb = (uint64_t)H * 2, rowy = (uint64_t)H * 4;
  const int* offsets = reinterpret_cast<const int*>(base + L.offsets);
  const int cap_grid = 4 * ctx->num_sms;
  {
    rl::PhaseTimer pt(ctx, st, RIALLM_PHASE_DISPATCH);
    EP_NCCL(ctx, n.AllGather(base + L.counts, loc + pl.cmat, E, ncclInt32, static_cast<ncclComm_t>(ctx->ep_comm), st),
            "ncclAllGather(counts)");
    ep_peer_plan_kernel<<<1, 32, 0, st>>>(a);
    const int gd = std::max(1, std::min((P + 7) / 8, cap_grid));
    ep_peer_dispatch_kernel<<<gd, 256, 0, st>>>(a, base + L.x_perm, offsets, P, rowb);
    ep_peer_wait_kernel<<<1, 32, 0, st>>>(a, kArrX, 0);
    EP_CUDA(ctx, cudaGetLastError(), "peer dispatch");
    ctx->launches += 3;
  }
  rl::TcGemmArgs g{};
  g.w = w->gate_up_proj;
  g.K = H;
  g.rows_per_expert = 2 * I;
  g.a1_offset = I;
  g.m_step = 128;
  g.m_tiles = I / 128;
  g.b = sym + pl.xr;
  g.P = pl.cap_x;
  g.counts = reinterpret_cast<const int*>(loc + pl.ecnt);
  g.offsets = reinterpret_cast<const int*>(loc + pl.eoff);
  g.E = EL;
  g.swiglu = true;
  g.h_pair_perm = w->down_proj.qtype == RIALLM_COMPRESSION_FOUR_BIT;
  g.h_out = reinterpret_cast<uint16_t*>(loc + pl.hr);
  g.ld_out = I;
  g.status = ctx->d_status;
  g.max_pairs_per_expert = pl.maxp;
  g.sk_ws = reinterpret_cast<float*>(loc + pl.skw);
  g.sk_flags = reinterpret_cast<int*>(base + L.sync + rl::kSkFlagsOffset);
  g.pdl = false;
  g.flag_wait_ns = ctx->flag_wait_ns;
  rl::TcGemmArgs d = g;
  d.w = w->down_proj;
  d.K = I;
  d.rows_per_expert = H;
  d.a1_offset = 128;
  d.m_step = 256;
  d.m_tiles = H / 256;
  d.b = loc + pl.hr;
  d.swiglu = false;
  d.h_pair_perm = false;
  d.h_out = nullptr;
  d.y_out = reinterpret_cast<float*>(loc + pl.yr);
  d.ld_out = H;
  d.pdl = false;  // follows the free_x signal, not the gate_up launch
  {
    rl::PhaseTimer pt(ctx, st, RIALLM_PHASE_GATE_UP);
    EP_CUDA(ctx, rl::launch_tc_gemm(g, ctx->num_sms, st), "expert gate_up (tcgen05)");
    ctx->launches += 1;
  }
  // The rows received this call are consumed: the senders may overwrite
  // them in the next call.
  ep_peer_signal_kernel<<<1, 32, 0, st>>>(a, kFreeX);
  EP_CUDA(ctx, cudaGetLastError(), "peer free signal");
  ctx->launches += 1;
  {
    rl::PhaseTimer pt(ctx, st, RIALLM_PHASE_DOWN);
    EP_CUDA(ctx, rl::launch_tc_gemm(d, ctx->num_sms, st), "expert down (tcgen05)");
    ctx->launches += 1;
  }
  {
    rl::PhaseTimer pt(ctx, st, RIALLM_PHASE_RETURN);
    ep_peer_wait_kernel<<<1, 32, 0, st>>>(a, kFreeY, 1);
    const int gr = std::max(1, std::min((pl.cap_x + 7) / 8, cap_grid));
    ep_peer_return_kernel<<<gr, 256, 0, st>>>(a, rowy);
    ep_peer_wait_kernel<<<1, 32, 0, st>>>(a, kArrY, 0);
    EP_CUDA(ctx, cudaGetLastError(), "peer return");
    ctx->launches += 3;
  }
  {
    rl::PhaseTimer pt(ctx, st, RIALLM_PHASE_COMBINE);
    EP_CUDA(ctx, rl::launch_combine(reinterpret_cast<const float*>(sym + pl.ret),
                                    reinterpret_cast<const int*>(base + L.inv_pos),
                                    reinterpret_cast<const int*>(base + L.topk_idx),
                                    reinterpret_cast<const float*>(base + L.topk_w), T, k, H, nullptr, nullptr, out,
                                    true, (flags & RIALLM_MOE_ADD_TO_OUT) != 0, st, 0, 1 << 30, true),
            "combine");
    ctx->launches += 1;
  }
  // This call's returns are consumed: the expert ranks may overwrite them.
  ep_peer_signal_kernel<<<1, 32, 0, st>>>(a, kFreeY);
  EP_CUDA(ctx, cudaGetLastError(), "peer free signal");
  ctx->launches += 1;
  return RIALLM_OK;
}

static void peer_teardown_ctx(riallm_ctx* ctx) { peer_teardown(ctx); }
