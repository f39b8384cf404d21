// noalloc.cu -- a MoE block entry point that never allocates device memory.
//
// Who needs it: code that runs where cudaMalloc is not available or not
// allowed -- for example a host that hands this library only pre-planned
// device memory, a real-time loop that must not call into the allocator
// (cudaMalloc can synchronize the device and its latency is unbounded), or a
// plugin host whose own allocator owns all device memory. Such callers can
// pass their inputs and outputs but cannot let the library grow a scratch
// arena, and they cannot create a riallm_ctx (creating one allocates).
//
// How: the scratch buffers of one block call (router weights, routing
// results, permutation, permuted activations, SwiGLU product, expert
// outputs) live in one file-scope __device__ array of kNoAllocScratchBytes.
// Every GPU that loads the library holds that array until the process exits.
// The host cannot use the array's name as a device address (on the host it
// is only a stand-in symbol), so the first call on each device looks the
// address up with cudaGetSymbolAddress while that device is current and
// caches it; that first call should therefore happen before any stream
// capture. All calls share the one array and it keeps the last call's
// contents: calls that overlap on the GPU (other streams, other host
// threads) race on it and must be serialized by the caller.
#include <cuda_runtime.h>

#include <mutex>

#include "internal.h"

constexpr uint64_t kNoAllocScratchBytes = 24ull << 20;  // 24 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ __align__(256) int g_noalloc_status;

namespace {

struct DeviceSlot {
  std::mutex mu;
  bool ready = false;
  unsigned char* scratch = nullptr;
  int* status = nullptr;
  int num_sms = 0;
};
constexpr int kMaxDevices = 64;
DeviceSlot g_slots[kMaxDevices];

// Per-device set-up with that device current: the device addresses of the
// scratch array and the status word, and the SM count. Only a successful
// set-up is kept; a failed one (for example a first call made inside a
// stream capture, where the look-up is not allowed) is tried again on the
// next call.
int device_setup(int dev, DeviceSlot** out) {
  if (dev < 0 || dev >= kMaxDevices) return RIALLM_ERR_CONFIG;
  DeviceSlot& s = g_slots[dev];
  std::lock_guard<std::mutex> lock(s.mu);
  if (!s.ready) {
    void* p = nullptr;
    void* q = nullptr;
    int sms = 0;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess ||
        cudaGetSymbolAddress(&q, g_noalloc_status) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();  // reset the runtime's last-error state; the next call retries
      return RIALLM_ERR_CUDA;
    }
    s.scratch = static_cast<unsigned char*>(p);
    s.status = static_cast<int*>(q);
    s.num_sms = sms;
    s.ready = true;
  }
  *out = &s;
  return RIALLM_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// The same checks, in the same order and with the same status codes, as
// the regular entry point applies to an expert tensor: a missing tensor is
// RIALLM_ERR_MODEL_LOADING, a wrong element count RIALLM_ERR_CONFIG, an
// unquantized or malformed one RIALLM_ERR_QUANTIZATION, unaligned buffers
// RIALLM_ERR_INVALID. need_quantized is false for the router weight, which
// may also be float32.
int check_tensor(const riallm_qtensor& t, uint64_t numel, bool need_quantized) {
  if (!t.data) return RIALLM_ERR_MODEL_LOADING;
  if (t.numel != numel) return RIALLM_ERR_CONFIG;
  if (t.qtype == RIALLM_COMPRESSION_NONE) {
    if (need_quantized) return RIALLM_ERR_QUANTIZATION;
    return aligned16(t.data) ? RIALLM_OK : RIALLM_ERR_INVALID;
  }
  if (t.qtype != RIALLM_COMPRESSION_FOUR_BIT && t.qtype != RIALLM_COMPRESSION_EIGHT_BIT)
    return RIALLM_ERR_QUANTIZATION;
  if (t.block_size != (t.qtype == RIALLM_COMPRESSION_FOUR_BIT ? 64 : 128)) return RIALLM_ERR_QUANTIZATION;
  if (!t.scales || !t.zero_points) return RIALLM_ERR_QUANTIZATION;
  if (!aligned16(t.data) || !aligned16(t.scales) || !aligned16(t.zero_points)) return RIALLM_ERR_INVALID;
  return RIALLM_OK;
}

}  // namespace

extern "C" int32_t riallm_cuda_moe_forward_noalloc(const riallm_moe_weights* w, const void* x,
                                                   void* out, int32_t T, int32_t H, int32_t I,
                                                   int32_t E, int32_t k, uint32_t flags,
                                                   void* stream) {
  if (!w) return RIALLM_ERR_INVALID;
  if (T < 0 || H <= 0 || I <= 0 || E <= 0 || k <= 0 || E > 256 || k > 16 || k > E) return RIALLM_ERR_CONFIG;
  if (H % 256 != 0 || I % 256 != 0) return RIALLM_ERR_CONFIG;
  if (w->shared_gate_proj.data != nullptr) return RIALLM_ERR_CONFIG;  // routed experts only
  if (int rc = check_tensor(w->gate, (uint64_t)E * H, false)) return rc;
  if (int rc = check_tensor(w->gate_up_proj, (uint64_t)E * 2 * I * H, true)) return rc;
  if (int rc = check_tensor(w->down_proj, (uint64_t)E * H * I, true)) return rc;
  if (T == 0) return RIALLM_OK;
  if (!x || !out || !aligned16(x) || !aligned16(out)) return RIALLM_ERR_INVALID;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RIALLM_ERR_CUDA;
  DeviceSlot* slot = nullptr;
  if (int rc = device_setup(dev, &slot)) return rc;

  // The whole scratch layout of one bf16 block call must fit the array;
  // when the expert GEMM's split-tile workspace does not fit as well, the
  // GEMM runs whole tiles per CTA instead.
  rl::MoeLayout L = rl::moe_layout(T, H, I, E, k, RIALLM_DTYPE_BF16, 0, slot->num_sms);
  if (L.total > kNoAllocScratchBytes) L = rl::moe_layout(T, H, I, E, k, RIALLM_DTYPE_BF16, 0, slot->num_sms, false);
  if (L.total > kNoAllocScratchBytes) return RIALLM_ERR_MEMORY;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* base = reinterpret_cast<char*>(slot->scratch);
  const int P = T * k;
  // The counters in the layout's first kSyncBytes (the router's completion
  // counter, the expert GEMM's split-tile counters) must read zero when the
  // call starts. A completed call leaves them at zero, but one that stopped
  // early (an expired device wait) may not, so they are cleared on every
  // call. Every other buffer is fully written before it is read within the
  // call. The status word is not cleared here: it keeps any call's timeout
  // until riallm_cuda_moe_forward_noalloc_sync reports and clears it.
  if (cudaMemsetAsync(base + L.sync, 0, rl::kSyncBytes, st) != cudaSuccess) return RIALLM_ERR_CUDA;
  int* topk_idx = reinterpret_cast<int*>(base + L.topk_idx);
  float* topk_w = reinterpret_cast<float*>(base + L.topk_w);
  int* counts = reinterpret_cast<int*>(base + L.counts);
  int* offsets = reinterpret_cast<int*>(base + L.offsets);
  int* perm = reinterpret_cast<int*>(base + L.perm_pair);
  int* inv = reinterpret_cast<int*>(base + L.inv_pos);
  rl::RouterArgs ra{};
  ra.x = x;
  ra.x_bf16 = 1;
  ra.gdata = w->gate.data;
  ra.gscales = w->gate.scales;
  ra.gzeros = w->gate.zero_points;
  ra.n_scales = w->gate.n_scales;
  ra.n_zeros = w->gate.n_zero_points;
  ra.T = T;
  ra.H = H;
  ra.E = E;
  ra.k = k;
  ra.topk_idx = topk_idx;
  ra.topk_w = topk_w;
  ra.counts = counts;
  ra.offsets = offsets;
  ra.perm_pair = perm;
  ra.inv_pos = inv;
  ra.done = reinterpret_cast<unsigned*>(base + L.sync);
  ra.cta_base = reinterpret_cast<int*>(base + L.cta_base);
  if (rl::launch_router(ra, w->gate.qtype, st) != cudaSuccess ||
      rl::launch_gather(x, true, perm, k, P, H, base + L.x_perm,
                        w->gate_up_proj.qtype == RIALLM_COMPRESSION_FOUR_BIT, st) != cudaSuccess)
    return RIALLM_ERR_CUDA;

  rl::TcGemmArgs g{};
  g.w = w->gate_up_proj;
  g.K = H;
  g.rows_per_expert = 2 * I;
  g.a1_offset = I;
  g.m_step = 128;
  g.m_tiles = I / 128;
  g.b = base + L.x_perm;
  g.P = P;
  g.counts = counts;
  g.offsets = offsets;
  g.E = E;
  g.swiglu = true;
  g.h_pair_perm = w->down_proj.qtype == RIALLM_COMPRESSION_FOUR_BIT;
  g.h_out = reinterpret_cast<uint16_t*>(base + L.h_perm);
  g.ld_out = I;
  g.status = slot->status;
  g.max_pairs_per_expert = T;
  g.sk_ws = L.sk_ws ? reinterpret_cast<float*>(base + L.sk_ws) : nullptr;
  g.sk_flags = reinterpret_cast<int*>(base + L.sync + rl::kSkFlagsOffset);
  g.pdl = true;  // follows the gather
  if (rl::launch_tc_gemm(g, slot->num_sms, st) != cudaSuccess) return RIALLM_ERR_CUDA;
  rl::TcGemmArgs d{};
  d.w = w->down_proj;
  d.K = I;
  d.rows_per_expert = H;
  d.a1_offset = 128;
  d.m_step = 256;
  d.m_tiles = H / 256;
  d.b = base + L.h_perm;
  d.P = P;
  d.counts = counts;
  d.offsets = offsets;
  d.E = E;
  d.swiglu = false;
  d.y_out = reinterpret_cast<float*>(base + L.y_perm);
  d.ld_out = H;
  d.status = slot->status;
  d.max_pairs_per_expert = T;
  d.sk_ws = L.sk_ws ? reinterpret_cast<float*>(base + L.sk_ws) : nullptr;
  d.sk_flags = reinterpret_cast<int*>(base + L.sync + rl::kSkFlagsOffset);
  d.pdl = true;  // follows the gate_up GEMM
  if (rl::launch_tc_gemm(d, slot->num_sms, st) != cudaSuccess) return RIALLM_ERR_CUDA;
  if (rl::launch_combine(reinterpret_cast<float*>(base + L.y_perm), inv, topk_idx, topk_w, T, k, H, nullptr,
                         nullptr, out, true, (flags & RIALLM_MOE_ADD_TO_OUT) != 0, st, 0, 1 << 30,
                         true) != cudaSuccess)
    return RIALLM_ERR_CUDA;
  return RIALLM_OK;
}

extern "C" int32_t riallm_cuda_moe_forward_noalloc_sync(void* stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RIALLM_ERR_CUDA;
  DeviceSlot* slot = nullptr;
  if (int rc = device_setup(dev, &slot)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return RIALLM_ERR_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, slot->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return RIALLM_ERR_CUDA;
  if (v == 0) return RIALLM_OK;
  if (cudaMemsetAsync(slot->status, 0, sizeof(int), st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
    return RIALLM_ERR_CUDA;
  return v;
}
