// api.cu -- the extern "C" entry points of libriallm_cuda (include/riallm_cuda.h).
//
// Orchestrates one MoE block call (src/model.rs:751-818) as a fixed sequence
// of launches on the caller's stream, with no host synchronisation:
//   router (router weight decoded on the fly, softmax, stable top-k, and the
//   counting sort of the token-expert pairs in its last CTA) -> gather
//   tokens -> expert GEMMs (tcgen05 for bf16 activations, CUDA cores for
//   float32) -> [shared expert] -> weighted combine. The small kernels and
//   the tcgen05 GEMMs use programmatic dependent launch, and at decode sizes
//   the gate_up GEMM prefetches the down GEMM's first weight stages into L2.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "internal.h"

using rl::MoeLayout;

namespace {

int set_err(riallm_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}

int cuda_err(riallm_ctx* ctx, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return RIALLM_OK;
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  if (e == cudaErrorMemoryAllocation) return set_err(ctx, RIALLM_ERR_MEMORY, m);
  return set_err(ctx, RIALLM_ERR_CUDA, m);
}

#define RL_CUDA(ctx, call, what)                 \
  do {                                           \
    cudaError_t _e = (call);                     \
    if (_e != cudaSuccess) return cuda_err(ctx, _e, what); \
  } while (0)

inline uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Checks a QuantizedTensor descriptor against its expected element count.
int check_qtensor(riallm_ctx* ctx, const riallm_qtensor& t, uint64_t numel, const char* name,
                  bool need_quantized) {
  if (t.data == nullptr) return set_err(ctx, RIALLM_ERR_MODEL_LOADING, std::string("Tensor not found: ") + name);
  if (t.numel != numel)
    return set_err(ctx, RIALLM_ERR_CONFIG, std::string(name) + ": numel " + std::to_string(t.numel) +
                                               " != expected " + std::to_string(numel));
  if (t.qtype == RIALLM_COMPRESSION_NONE) {
    if (need_quantized)
      return set_err(ctx, RIALLM_ERR_QUANTIZATION, std::string(name) + ": expert weights must be FourBit or EightBit");
    return RIALLM_OK;
  }
  if (t.qtype != RIALLM_COMPRESSION_FOUR_BIT && t.qtype != RIALLM_COMPRESSION_EIGHT_BIT)
    return set_err(ctx, RIALLM_ERR_QUANTIZATION, std::string(name) + ": unknown qtype");
  const int want_bs = t.qtype == RIALLM_COMPRESSION_FOUR_BIT ? 64 : 128;
  if (t.block_size != want_bs)
    return set_err(ctx, RIALLM_ERR_QUANTIZATION,
                   std::string(name) + ": block_size " + std::to_string(t.block_size) + " unsupported");
  if (t.scales == nullptr || t.zero_points == nullptr)
    return set_err(ctx, RIALLM_ERR_QUANTIZATION, std::string(name) + ": missing scales/zero_points");
  if (!aligned16(t.data) || !aligned16(t.scales) || !aligned16(t.zero_points))
    return set_err(ctx, RIALLM_ERR_INVALID, std::string(name) + ": device buffers must be 16-byte aligned");
  return RIALLM_OK;
}

int ensure_arena(riallm_ctx* ctx, uint64_t bytes) {
  if (ctx->arena_bytes >= bytes) return RIALLM_OK;
  if (ctx->arena) {
    // Kept, not freed: graphs that captured earlier calls still point at it.
    ctx->retired_arenas.push_back(ctx->arena);
    ctx->arena = nullptr;
    ctx->arena_bytes = 0;
  }
  const uint64_t sz = align_up(bytes, 2u << 20);
  RL_CUDA(ctx, cudaMalloc(&ctx->arena, sz), "cudaMalloc(arena)");
  ctx->arena_bytes = sz;
  // The layout's first kSyncBytes are counters that must read zero before
  // the first call (each call leaves them at zero).
  RL_CUDA(ctx, cudaMemset(ctx->arena, 0, rl::kSyncBytes), "cudaMemset(arena)");
  RL_CUDA(ctx, cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  return RIALLM_OK;
}

int set_device(riallm_ctx* ctx) {
  RL_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  return RIALLM_OK;
}


}  // namespace

namespace rl {

MoeLayout moe_layout(int T, int H, int I, int E, int k, int act_dtype, int shared_I, int num_sms,
                     bool with_sk) {
  MoeLayout L{};
  const uint64_t P = (uint64_t)T * k;
  const uint64_t a = 1024;
  const uint64_t esz = act_dtype == RIALLM_DTYPE_BF16 ? 2 : 4;
  uint64_t o = 0;
  auto take = [&](uint64_t bytes) {
    uint64_t r = o;
    o = align_up(o + bytes, a);
    return r;
  };
  L.sync = take(kSyncBytes);
  L.sk_ws = (with_sk && act_dtype == RIALLM_DTYPE_BF16) ? take(tc_sk_ws_bytes(num_sms, T)) : 0;
  L.topk_idx = take(P * 4);
  L.topk_w = take(P * 4);
  L.counts = take((uint64_t)E * 4);
  L.offsets = take((uint64_t)(E + 1) * 4);
  L.perm_pair = take(P * 4);
  L.inv_pos = take(P * 4);
  L.cta_base = take((int64_t)P > kSortOneCta ? router_cta_bytes(T, H, E) : 0);
  L.gate_f32_bytes = router_tile_tokens(T, H) > 1 ? (uint64_t)E * H * 4 : 0;
  L.gate_f32 = take(L.gate_f32_bytes);
  L.x_perm = take(P * H * esz);
  L.h_perm = take(P * I * esz);
  L.y_perm = take(P * H * 4);
  L.proj = act_dtype == RIALLM_DTYPE_BF16 ? take(0) : take(P * 2 * (uint64_t)I * 4);
  if (shared_I > 0) {
    L.sh_g = take((uint64_t)T * shared_I * 4);
    L.sh_u = take((uint64_t)T * shared_I * 4);
    L.sh_h = take((uint64_t)T * shared_I * esz);
    L.sh_y = take((uint64_t)T * H * 4);
    L.sh_gate = take((uint64_t)T * 4);
  }
  L.total = o + a;
  return L;
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                              CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                              CUtensorMapFloatOOBfill);

CUresult encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                              uint64_t dim0, uint64_t dim1, uint64_t row_stride_bytes,
                              uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle) {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  if (!fn) return CUDA_ERROR_NOT_FOUND;
  const cuuint64_t dims[2] = {dim0, dim1};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box0, box1};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace rl

extern "C" {

int32_t riallm_cuda_abi_version(void) { return RIALLM_CUDA_ABI_VERSION; }

int32_t riallm_cuda_ctx_create(int32_t device, riallm_ctx** out) {
  if (!out) return RIALLM_ERR_INVALID;
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || device < 0 || device >= n) return RIALLM_ERR_CONFIG;
  riallm_ctx* ctx = new riallm_ctx();
  ctx->device = device;
  if (cudaSetDevice(device) != cudaSuccess) {
    delete ctx;
    return RIALLM_ERR_CUDA;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    delete ctx;
    return RIALLM_ERR_CUDA;
  }
  if (prop.major != 10) {
    delete ctx;
    return RIALLM_ERR_CONFIG;  // sm_100a only
  }
  ctx->num_sms = prop.multiProcessorCount;
  if (cudaMalloc(&ctx->d_status, sizeof(int)) != cudaSuccess ||
      cudaMemset(ctx->d_status, 0, sizeof(int)) != cudaSuccess ||
      cudaMalloc(&ctx->attn_ws, rl::attn_ws_bytes(ctx->num_sms)) != cudaSuccess ||
      cudaMemset(ctx->attn_ws, 0, rl::kAttnCounterBytes) != cudaSuccess) {
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->attn_ws) cudaFree(ctx->attn_ws);
    delete ctx;
    return RIALLM_ERR_MEMORY;
  }
  *out = ctx;
  return RIALLM_OK;
}

int32_t riallm_cuda_ctx_destroy(riallm_ctx* ctx) {
  if (!ctx) return RIALLM_ERR_INVALID;
  riallm_cuda_ep_destroy(ctx);
  cudaSetDevice(ctx->device);
  if (ctx->arena) cudaFree(ctx->arena);
  for (void* a : ctx->retired_arenas) cudaFree(a);
  if (ctx->d_status) cudaFree(ctx->d_status);
  if (ctx->attn_ws) cudaFree(ctx->attn_ws);
  for (auto& pe : ctx->pending) {
    cudaEventDestroy(pe.start);
    cudaEventDestroy(pe.stop);
  }
  for (cudaEvent_t e : ctx->event_pool) cudaEventDestroy(e);
  delete ctx;
  return RIALLM_OK;
}

const char* riallm_cuda_last_error(const riallm_ctx* ctx) {
  return ctx ? ctx->last_error.c_str() : "null context";
}

int32_t riallm_cuda_alloc(riallm_ctx* ctx, uint64_t bytes, void** dptr) {
  if (!ctx || !dptr) return RIALLM_ERR_INVALID;
  if (int s = set_device(ctx)) return s;
  RL_CUDA(ctx, cudaMalloc(dptr, bytes), "cudaMalloc");
  return RIALLM_OK;
}

int32_t riallm_cuda_free(riallm_ctx* ctx, void* dptr) {
  if (!ctx) return RIALLM_ERR_INVALID;
  RL_CUDA(ctx, cudaFree(dptr), "cudaFree");
  return RIALLM_OK;
}

int32_t riallm_cuda_host_alloc_pinned(riallm_ctx* ctx, uint64_t bytes, void** hptr) {
  if (!ctx || !hptr) return RIALLM_ERR_INVALID;
  RL_CUDA(ctx, cudaHostAlloc(hptr, bytes, cudaHostAllocDefault), "cudaHostAlloc");
  return RIALLM_OK;
}

int32_t riallm_cuda_host_free_pinned(riallm_ctx* ctx, void* hptr) {
  if (!ctx) return RIALLM_ERR_INVALID;
  RL_CUDA(ctx, cudaFreeHost(hptr), "cudaFreeHost");
  return RIALLM_OK;
}

int32_t riallm_cuda_memcpy_h2d_async(riallm_ctx* ctx, void* dst, const void* src, uint64_t bytes,
                                     void* stream) {
  if (!ctx) return RIALLM_ERR_INVALID;
  RL_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream),
          "cudaMemcpyAsync(H2D)");
  return RIALLM_OK;
}

int32_t riallm_cuda_memcpy_d2h_async(riallm_ctx* ctx, void* dst, const void* src, uint64_t bytes,
                                     void* stream) {
  if (!ctx) return RIALLM_ERR_INVALID;
  RL_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream),
          "cudaMemcpyAsync(D2H)");
  return RIALLM_OK;
}

int32_t riallm_cuda_stream_synchronize(riallm_ctx* ctx, void* stream) {
  if (!ctx) return RIALLM_ERR_INVALID;
  RL_CUDA(ctx, cudaStreamSynchronize((cudaStream_t)stream), "cudaStreamSynchronize");
  int st = 0;
  RL_CUDA(ctx, cudaMemcpy(&st, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost), "status read");
  if (st != 0) {
    cudaMemset(ctx->d_status, 0, sizeof(int));
    // An aborted kernel may leave the arena's call counters non-zero.
    if (ctx->arena) cudaMemset(ctx->arena, 0, rl::kSyncBytes);
    cudaDeviceSynchronize();
    return set_err(ctx, st, "a bounded device-side wait expired (kernel aborted)");
  }
  return RIALLM_OK;
}

int32_t riallm_cuda_memory_stats(riallm_ctx* ctx, uint64_t* free_bytes, uint64_t* total_bytes) {
  if (!ctx || !free_bytes || !total_bytes) return RIALLM_ERR_INVALID;
  if (int s = set_device(ctx)) return s;
  size_t f = 0, t = 0;
  RL_CUDA(ctx, cudaMemGetInfo(&f, &t), "cudaMemGetInfo");
  *free_bytes = f;
  *total_bytes = t;
  return RIALLM_OK;
}

uint64_t riallm_quant_num_blocks(int32_t qtype, uint64_t numel) {
  if (qtype == RIALLM_COMPRESSION_FOUR_BIT) return (numel + 63) / 64;
  if (qtype == RIALLM_COMPRESSION_EIGHT_BIT) return (numel + 127) / 128;
  return 0;
}

uint64_t riallm_quant_data_bytes(int32_t qtype, uint64_t numel) {
  if (qtype == RIALLM_COMPRESSION_FOUR_BIT) return (numel + 1) / 2;
  if (qtype == RIALLM_COMPRESSION_EIGHT_BIT) return numel;
  return numel * 4;
}

int32_t riallm_cuda_quantize(riallm_ctx* ctx, int32_t qtype, const float* src, uint64_t numel,
                             uint8_t* data, float* scales, float* zero_points, void* stream) {
  if (!ctx) return RIALLM_ERR_INVALID;
  if (qtype != RIALLM_COMPRESSION_FOUR_BIT && qtype != RIALLM_COMPRESSION_EIGHT_BIT)
    return set_err(ctx, RIALLM_ERR_QUANTIZATION, "No compression specified");
  if (!src || !data || !scales || !zero_points) return set_err(ctx, RIALLM_ERR_INVALID, "null buffer");
  if (numel == 0) return RIALLM_OK;
  if (int s = set_device(ctx)) return s;
  RL_CUDA(ctx, rl::launch_quantize(qtype, src, numel, data, scales, zero_points, ctx->num_sms,
                                   (cudaStream_t)stream),
          "quantize launch");
  return RIALLM_OK;
}

int32_t riallm_cuda_dequantize(riallm_ctx* ctx, const riallm_qtensor* t, int32_t mode, void* dst,
                               int32_t dst_dtype, void* stream) {
  if (!ctx || !t || !dst) return RIALLM_ERR_INVALID;
  if (t->qtype != RIALLM_COMPRESSION_NONE && t->qtype != RIALLM_COMPRESSION_FOUR_BIT &&
      t->qtype != RIALLM_COMPRESSION_EIGHT_BIT)
    return set_err(ctx, RIALLM_ERR_QUANTIZATION, "unknown qtype");
  if (t->qtype == RIALLM_COMPRESSION_NONE && mode == RIALLM_DEQUANT_REFERENCE)
    return set_err(ctx, RIALLM_ERR_QUANTIZATION, "Tensor is not quantized");
  if (t->qtype != RIALLM_COMPRESSION_NONE && (t->block_size <= 0 || (t->qtype == RIALLM_COMPRESSION_FOUR_BIT && (t->block_size & 1))))
    return set_err(ctx, RIALLM_ERR_QUANTIZATION, "block_size must be positive (and even for NF4)");
  if (t->numel == 0) return RIALLM_OK;
  if (int s = set_device(ctx)) return s;
  RL_CUDA(ctx, rl::launch_dequant(*t, mode, dst, dst_dtype, ctx->num_sms, (cudaStream_t)stream),
          "dequantize launch");
  return RIALLM_OK;
}

static int check_shapes(riallm_ctx* ctx, int T, int H, int I, int E, int k) {
  if (T < 0 || H <= 0 || I <= 0 || E <= 0 || k <= 0)
    return set_err(ctx, RIALLM_ERR_CONFIG, "non-positive MoE dimension");
  if (E > 256 || k > 16 || k > E)
    return set_err(ctx, RIALLM_ERR_CONFIG, "need E <= 256, k <= 16, k <= E");
  if (H % 256 != 0 || I % 256 != 0)
    return set_err(ctx, RIALLM_ERR_CONFIG, "need hidden % 256 == 0 and intermediate % 256 == 0");
  if ((int64_t)T * k > (1ll << 24)) return set_err(ctx, RIALLM_ERR_CONFIG, "too many tokens");
  return RIALLM_OK;
}

int32_t riallm_cuda_moe_reserve(riallm_ctx* ctx, int32_t T, int32_t H, int32_t I, int32_t E,
                                int32_t k, int32_t act_dtype) {
  if (!ctx) return RIALLM_ERR_INVALID;
  if (int s = check_shapes(ctx, T, H, I, E, k)) return s;
  if (int s = set_device(ctx)) return s;
  MoeLayout L = rl::moe_layout(T, H, I, E, k, act_dtype, 0, ctx->num_sms);
  return ensure_arena(ctx, L.total);
}

static int route_into(riallm_ctx* ctx, const riallm_qtensor& gate, const void* x, int T, int H, int E,
                      int k, bool bf16, char* base, const MoeLayout& L, cudaStream_t st) {
  if (gate.qtype == RIALLM_COMPRESSION_NONE && !aligned16(gate.data))
    return set_err(ctx, RIALLM_ERR_INVALID, "mlp.gate.weight: device buffer must be 16-byte aligned");
  rl::RouterArgs a{};
  a.x = x;
  a.x_bf16 = bf16 ? 1 : 0;
  a.gdata = gate.data;
  a.gscales = gate.scales;
  a.gzeros = gate.zero_points;
  a.n_scales = gate.n_scales;
  a.n_zeros = gate.n_zero_points;
  a.T = T;
  a.H = H;
  a.E = E;
  a.k = k;
  a.topk_idx = (int*)(base + L.topk_idx);
  a.topk_w = (float*)(base + L.topk_w);
  a.counts = (int*)(base + L.counts);
  a.offsets = (int*)(base + L.offsets);
  a.perm_pair = (int*)(base + L.perm_pair);
  a.inv_pos = (int*)(base + L.inv_pos);
  a.done = (unsigned*)(base + L.sync);
  a.cta_base = (int*)(base + L.cta_base);
  if ((int64_t)T * k > rl::kSortOneCta)
    RL_CUDA(ctx, cudaMemsetAsync(a.cta_base, 0, rl::router_cta_bytes(T, H, E), st), "router group counts");
  int qtype = gate.qtype;
  if (qtype != RIALLM_COMPRESSION_NONE && L.gate_f32_bytes) {
    // Token-tiled calls decode the router weight once (the reference's
    // decode, src/quantization.rs:45-95, the same float32 values the router
    // would decode per CTA), so every CTA reads float32 rows: the per-CTA
    // decode was a third of the router's instructions.
    float* gf = reinterpret_cast<float*>(base + L.gate_f32);
    RL_CUDA(ctx, rl::launch_dequant(gate, 0, gf, RIALLM_DTYPE_F32, ctx->num_sms, st), "router weight decode");
    ctx->launches += 1;
    a.gdata = gf;
    a.gscales = a.gzeros = nullptr;
    a.n_scales = a.n_zeros = 0;
    qtype = RIALLM_COMPRESSION_NONE;
  }
  a.gate_v8 = qtype == RIALLM_COMPRESSION_NONE && (reinterpret_cast<uintptr_t>(a.gdata) & 31) == 0 ? 1 : 0;
  RL_CUDA(ctx, rl::launch_router(a, qtype, st), "router");
  return RIALLM_OK;
}

int32_t riallm_cuda_moe_route(riallm_ctx* ctx, const riallm_qtensor* gate, const void* x, int32_t T,
                              int32_t H, int32_t E, int32_t k, int32_t act_dtype, int32_t* topk_idx,
                              float* topk_w, int32_t* counts, int32_t* offsets, int32_t* perm_pair,
                              void* stream) {
  if (!ctx || !gate) return RIALLM_ERR_INVALID;
  if ((!x || !topk_idx) && T != 0) return set_err(ctx, RIALLM_ERR_INVALID, "null x/topk_idx");
  if (T < 0 || H <= 0 || E <= 0 || k <= 0 || E > 256 || k > 16 || k > E || H % 8 != 0)
    return set_err(ctx, RIALLM_ERR_CONFIG, "router shape out of range");
  if (int s = check_qtensor(ctx, *gate, (uint64_t)E * H, "mlp.gate.weight", false)) return s;
  if (T == 0) return RIALLM_OK;
  if (!aligned16(x)) return set_err(ctx, RIALLM_ERR_INVALID, "x must be 16-byte aligned");
  if (int s = set_device(ctx)) return s;
  const bool bf16 = act_dtype == RIALLM_DTYPE_BF16;
  MoeLayout L = rl::moe_layout(T, H, 256, E, k, act_dtype, 0, ctx->num_sms, false);
  if (int s = ensure_arena(ctx, L.total)) return s;
  char* base = (char*)ctx->arena;
  cudaStream_t st = (cudaStream_t)stream;
  if (int s = route_into(ctx, *gate, x, T, H, E, k, bf16, base, L, st)) return s;
  const uint64_t P = (uint64_t)T * k;
  RL_CUDA(ctx, cudaMemcpyAsync(topk_idx, base + L.topk_idx, P * 4, cudaMemcpyDeviceToDevice, st), "copy idx");
  if (topk_w)
    RL_CUDA(ctx, cudaMemcpyAsync(topk_w, base + L.topk_w, P * 4, cudaMemcpyDeviceToDevice, st), "copy w");
  if (counts)
    RL_CUDA(ctx, cudaMemcpyAsync(counts, base + L.counts, (uint64_t)E * 4, cudaMemcpyDeviceToDevice, st),
            "copy counts");
  if (offsets)
    RL_CUDA(ctx, cudaMemcpyAsync(offsets, base + L.offsets, (uint64_t)(E + 1) * 4, cudaMemcpyDeviceToDevice, st),
            "copy offsets");
  if (perm_pair)
    RL_CUDA(ctx, cudaMemcpyAsync(perm_pair, base + L.perm_pair, P * 4, cudaMemcpyDeviceToDevice, st),
            "copy perm");
  return RIALLM_OK;
}

int32_t riallm_cuda_moe_forward(riallm_ctx* ctx, const riallm_moe_weights* w, const void* x, void* out,
                                int32_t T, int32_t H, int32_t I, int32_t E, int32_t k, int32_t act_dtype,
                                uint32_t flags, void* stream) {
  if (!ctx || !w) return RIALLM_ERR_INVALID;
  if ((!x || !out) && T != 0) return set_err(ctx, RIALLM_ERR_INVALID, "null x/out");
  if (act_dtype != RIALLM_DTYPE_BF16 && act_dtype != RIALLM_DTYPE_F32)
    return set_err(ctx, RIALLM_ERR_CONFIG, "act_dtype must be F32 or BF16");
  if (int s = check_shapes(ctx, T, H, I, E, k)) return s;
  if (int s = check_qtensor(ctx, w->gate, (uint64_t)E * H, "mlp.gate.weight", false)) return s;
  if (int s = check_qtensor(ctx, w->gate_up_proj, (uint64_t)E * 2 * I * H, "mlp.experts.gate_up_proj", true)) return s;
  if (int s = check_qtensor(ctx, w->down_proj, (uint64_t)E * H * I, "mlp.experts.down_proj", true)) return s;
  const bool shared = w->shared_gate_proj.data != nullptr;
  const int Is = shared ? w->shared_intermediate : 0;
  if (shared) {
    if (Is <= 0) return set_err(ctx, RIALLM_ERR_CONFIG, "shared_intermediate must be positive");
    if (int s = check_qtensor(ctx, w->shared_gate_proj, (uint64_t)Is * H, "mlp.shared_expert.gate_proj.weight", false)) return s;
    if (int s = check_qtensor(ctx, w->shared_up_proj, (uint64_t)Is * H, "mlp.shared_expert.up_proj.weight", false)) return s;
    if (int s = check_qtensor(ctx, w->shared_down_proj, (uint64_t)H * Is, "mlp.shared_expert.down_proj.weight", false)) return s;
    if (int s = check_qtensor(ctx, w->shared_expert_gate, (uint64_t)H, "mlp.shared_expert_gate.weight", false)) return s;
  }
  if (T == 0) return RIALLM_OK;
  if (!aligned16(x) || !aligned16(out)) return set_err(ctx, RIALLM_ERR_INVALID, "x/out must be 16-byte aligned");
  if (int s = set_device(ctx)) return s;

  const bool bf16 = act_dtype == RIALLM_DTYPE_BF16;
  const int P = T * k;
  MoeLayout L = rl::moe_layout(T, H, I, E, k, act_dtype, Is, ctx->num_sms);
  if (int s = ensure_arena(ctx, L.total)) return s;
  char* base = (char*)ctx->arena;
  cudaStream_t st = (cudaStream_t)stream;

  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_ROUTE);
    if (int s = route_into(ctx, w->gate, x, T, H, E, k, bf16, base, L, st)) return s;
    ctx->launches += 1;
  }
  const int* counts = (const int*)(base + L.counts);
  const int* offsets = (const int*)(base + L.offsets);
  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_GATHER);
    RL_CUDA(ctx, rl::launch_gather(x, bf16, (const int*)(base + L.perm_pair), k, P, H, base + L.x_perm,
                                   bf16 && w->gate_up_proj.qtype == RIALLM_COMPRESSION_FOUR_BIT, st),
            "gather");
    ctx->launches += 1;
  }

  if (bf16) {
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
    g.h_out = (uint16_t*)(base + L.h_perm);
    g.ld_out = I;
    g.status = ctx->d_status;
    g.max_pairs_per_expert = T;
    g.sk_ws = L.sk_ws ? (float*)(base + L.sk_ws) : nullptr;
    g.sk_flags = (int*)(base + L.sync + rl::kSkFlagsOffset);
    g.pdl = true;  // follows the gather
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
    d.y_out = (float*)(base + L.y_perm);
    d.ld_out = H;
    d.status = ctx->d_status;
    d.max_pairs_per_expert = T;
    d.sk_ws = L.sk_ws ? (float*)(base + L.sk_ws) : nullptr;
    d.sk_flags = (int*)(base + L.sync + rl::kSkFlagsOffset);
    d.pdl = true;  // follows the gate_up GEMM
    g.next = &d;  // gate_up prefetches the down launch's first weight stages
    g.flag_wait_ns = d.flag_wait_ns = ctx->flag_wait_ns;
    if (ctx->expire_next_wait) {
      // Test hook: both launches' split-tile owners wait for a partial-sum
      // count no CTA reaches, so their bounded waits expire.
      g.flag_extra = d.flag_extra = 1 << 20;
      ctx->expire_next_wait = false;
    }
    {
      rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_GATE_UP);
      RL_CUDA(ctx, rl::launch_tc_gemm(g, ctx->num_sms, st), "expert gate_up (tcgen05)");
      ctx->launches += 1;
    }
    {
      rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_DOWN);
      RL_CUDA(ctx, rl::launch_tc_gemm(d, ctx->num_sms, st), "expert down (tcgen05)");
      ctx->launches += 1;
    }
  } else {
    float* proj = (float*)(base + L.proj);
    rl::GroupedF32Args g{};
    g.w = w->gate_up_proj;
    g.K = H;
    g.rows = 2 * I;
    g.rows_per_expert = 2 * I;
    g.row_offset = 0;
    g.x = base + L.x_perm;
    g.x_bf16 = false;
    g.y = proj;
    g.ldy = 2 * I;
    g.y_col0 = 0;
    g.counts = counts;
    g.offsets = offsets;
    g.E = E;
    g.P = P;
    g.round_w_bf16 = false;
    {
      rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_GATE_UP);
      RL_CUDA(ctx, rl::launch_grouped_f32(g, st), "expert gate_up (f32)");
      RL_CUDA(ctx, rl::launch_swiglu(proj, 2 * I, proj + I, 2 * I, base + L.h_perm, I, P, I, false, st),
              "swiglu");
      ctx->launches += 2;
    }
    rl::GroupedF32Args d = g;
    d.w = w->down_proj;
    d.K = I;
    d.rows = H;
    d.rows_per_expert = H;
    d.x = base + L.h_perm;
    d.y = (float*)(base + L.y_perm);
    d.ldy = H;
    {
      rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_DOWN);
      RL_CUDA(ctx, rl::launch_grouped_f32(d, st), "expert down (f32)");
      ctx->launches += 1;
    }
  }

  const float* shared_y = nullptr;
  const float* shared_gate = nullptr;
  if (shared) {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_SHARED);
    ctx->launches += 5;
    rl::GroupedF32Args s{};
    s.K = H;
    s.rows = Is;
    s.rows_per_expert = Is;
    s.row_offset = 0;
    s.x = x;
    s.x_bf16 = bf16;
    s.ldy = Is;
    s.counts = nullptr;
    s.P = T;
    s.E = 1;
    s.round_w_bf16 = bf16;
    s.w = w->shared_gate_proj;
    s.y = (float*)(base + L.sh_g);
    RL_CUDA(ctx, rl::launch_grouped_f32(s, st), "shared gate_proj");
    s.w = w->shared_up_proj;
    s.y = (float*)(base + L.sh_u);
    RL_CUDA(ctx, rl::launch_grouped_f32(s, st), "shared up_proj");
    RL_CUDA(ctx, rl::launch_swiglu((float*)(base + L.sh_g), Is, (float*)(base + L.sh_u), Is, base + L.sh_h,
                                   Is, T, Is, bf16, st),
            "shared swiglu");
    rl::GroupedF32Args sd = s;
    sd.w = w->shared_down_proj;
    sd.K = Is;
    sd.rows = H;
    sd.rows_per_expert = H;
    sd.x = base + L.sh_h;
    sd.y = (float*)(base + L.sh_y);
    sd.ldy = H;
    RL_CUDA(ctx, rl::launch_grouped_f32(sd, st), "shared down_proj");
    rl::GroupedF32Args sg = s;
    sg.w = w->shared_expert_gate;
    sg.rows = 1;
    sg.rows_per_expert = 1;
    sg.y = (float*)(base + L.sh_gate);
    sg.ldy = 1;
    sg.round_w_bf16 = false;
    RL_CUDA(ctx, rl::launch_grouped_f32(sg, st), "shared expert gate");
    shared_y = (const float*)(base + L.sh_y);
    shared_gate = (const float*)(base + L.sh_gate);
  }

  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_COMBINE);
    RL_CUDA(ctx, rl::launch_combine((const float*)(base + L.y_perm), (const int*)(base + L.inv_pos),
                                    (const int*)(base + L.topk_idx), (const float*)(base + L.topk_w), T, k, H,
                                    shared_y, shared_gate, out, bf16, (flags & RIALLM_MOE_ADD_TO_OUT) != 0, st,
                                    0, 1 << 30, bf16),
            "combine");
    ctx->launches += 1;
  }
  if (ctx->profiling) ctx->profiled_calls += 1;
  return RIALLM_OK;
}

int32_t riallm_cuda_moe_forward_ep(riallm_ctx* ctx, const riallm_moe_weights* w, const void* x,
                                   float* partial, int32_t T, int32_t H, int32_t I, int32_t E, int32_t k,
                                   int32_t e_begin, int32_t e_local, void* stream) {
  if (!ctx || !w) return RIALLM_ERR_INVALID;
  if ((!x || !partial) && T != 0) return set_err(ctx, RIALLM_ERR_INVALID, "null x/partial");
  if (int s = check_shapes(ctx, T, H, I, E, k)) return s;
  if (e_begin < 0 || e_local <= 0 || e_begin + e_local > E)
    return set_err(ctx, RIALLM_ERR_CONFIG, "expert range [e_begin, e_begin + e_local) outside [0, E)");
  if (w->shared_gate_proj.data != nullptr)
    return set_err(ctx, RIALLM_ERR_CONFIG, "expert-parallel calls take routed experts only");
  if (int s = check_qtensor(ctx, w->gate, (uint64_t)E * H, "mlp.gate.weight", false)) return s;
  if (int s = check_qtensor(ctx, w->gate_up_proj, (uint64_t)e_local * 2 * I * H, "mlp.experts.gate_up_proj", true))
    return s;
  if (int s = check_qtensor(ctx, w->down_proj, (uint64_t)e_local * H * I, "mlp.experts.down_proj", true)) return s;
  if (T == 0) return RIALLM_OK;
  if (!aligned16(x) || !aligned16(partial)) return set_err(ctx, RIALLM_ERR_INVALID, "x/partial must be 16-byte aligned");
  if (int s = set_device(ctx)) return s;
  const int P = T * k;
  MoeLayout L = rl::moe_layout(T, H, I, E, k, RIALLM_DTYPE_BF16, 0, ctx->num_sms);
  if (int s = ensure_arena(ctx, L.total)) return s;
  char* base = (char*)ctx->arena;
  cudaStream_t st = (cudaStream_t)stream;
  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_ROUTE);
    if (int s = route_into(ctx, w->gate, x, T, H, E, k, true, base, L, st)) return s;
    ctx->launches += 1;
  }
  // This rank's experts own the pair rows [offsets[e_begin], offsets[e_end]).
  const int* counts = (const int*)(base + L.counts) + e_begin;
  const int* offsets = (const int*)(base + L.offsets) + e_begin;
  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_GATHER);
    RL_CUDA(ctx, rl::launch_gather(x, true, (const int*)(base + L.perm_pair), k, P, H, base + L.x_perm,
                                   w->gate_up_proj.qtype == RIALLM_COMPRESSION_FOUR_BIT, st, offsets,
                                   offsets + e_local),
            "gather");
    ctx->launches += 1;
  }
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
  g.E = e_local;
  g.swiglu = true;
  g.h_pair_perm = w->down_proj.qtype == RIALLM_COMPRESSION_FOUR_BIT;
  g.h_out = (uint16_t*)(base + L.h_perm);
  g.ld_out = I;
  g.status = ctx->d_status;
  g.max_pairs_per_expert = T;
  g.sk_ws = L.sk_ws ? (float*)(base + L.sk_ws) : nullptr;
  g.sk_flags = (int*)(base + L.sync + rl::kSkFlagsOffset);
  g.pdl = true;  // follows the gather
  g.flag_wait_ns = ctx->flag_wait_ns;
  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_GATE_UP);
    RL_CUDA(ctx, rl::launch_tc_gemm(g, ctx->num_sms, st), "expert gate_up (tcgen05)");
    ctx->launches += 1;
  }
  rl::TcGemmArgs d = g;
  d.w = w->down_proj;
  d.K = I;
  d.rows_per_expert = H;
  d.a1_offset = 128;
  d.m_step = 256;
  d.m_tiles = H / 256;
  d.b = base + L.h_perm;
  d.swiglu = false;
  d.h_pair_perm = false;
  d.h_out = nullptr;
  d.y_out = (float*)(base + L.y_perm);
  d.ld_out = H;
  d.pdl = true;  // follows the gate_up GEMM
  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_DOWN);
    RL_CUDA(ctx, rl::launch_tc_gemm(d, ctx->num_sms, st), "expert down (tcgen05)");
    ctx->launches += 1;
  }
  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_COMBINE);
    RL_CUDA(ctx, rl::launch_combine((const float*)(base + L.y_perm), (const int*)(base + L.inv_pos),
                                    (const int*)(base + L.topk_idx), (const float*)(base + L.topk_w), T, k, H,
                                    nullptr, nullptr, partial, false, false, st, e_begin, e_begin + e_local,
                                    true),
            "combine (partial)");
    ctx->launches += 1;
  }
  if (ctx->profiling) ctx->profiled_calls += 1;
  return RIALLM_OK;
}

int32_t riallm_cuda_moe_forward_ep_a2a(riallm_ctx* ctx, const riallm_moe_weights* w, const void* x, void* out,
                                       int32_t T, int32_t H, int32_t I, int32_t E, int32_t k, uint32_t flags,
                                       void* stream) {
  if (!ctx || !w) return RIALLM_ERR_INVALID;
  if (!ctx->ep_comm) return set_err(ctx, RIALLM_ERR_CONFIG, "riallm_cuda_ep_init was not called on this context");
  if (T < 1) return set_err(ctx, RIALLM_ERR_CONFIG, "every rank calls with the same T >= 1");
  if (!x || !out) return set_err(ctx, RIALLM_ERR_INVALID, "null x/out");
  if (int s = check_shapes(ctx, T, H, I, E, k)) return s;
  const int W = ctx->ep_world;
  if (E % W) return set_err(ctx, RIALLM_ERR_CONFIG, "experts do not split evenly over the ranks");
  const int EL = E / W;
  if (w->shared_gate_proj.data != nullptr)
    return set_err(ctx, RIALLM_ERR_CONFIG, "expert-parallel calls take routed experts only");
  if (int s = check_qtensor(ctx, w->gate, (uint64_t)E * H, "mlp.gate.weight", false)) return s;
  if (int s = check_qtensor(ctx, w->gate_up_proj, (uint64_t)EL * 2 * I * H, "mlp.experts.gate_up_proj", true))
    return s;
  if (int s = check_qtensor(ctx, w->down_proj, (uint64_t)EL * H * I, "mlp.experts.down_proj", true)) return s;
  if (!aligned16(x) || !aligned16(out)) return set_err(ctx, RIALLM_ERR_INVALID, "x/out must be 16-byte aligned");
  if (int s = set_device(ctx)) return s;
  const int P = T * k;
  MoeLayout L = rl::moe_layout(T, H, I, E, k, RIALLM_DTYPE_BF16, 0, ctx->num_sms);
  if (int s = ensure_arena(ctx, L.total + rl_ep_extra_bytes(T, H, I, E, k, W, ctx->num_sms))) return s;
  char* base = (char*)ctx->arena;
  cudaStream_t st = (cudaStream_t)stream;
  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_ROUTE);
    if (int s = route_into(ctx, w->gate, x, T, H, E, k, true, base, L, st)) return s;
    ctx->launches += 1;
  }
  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_GATHER);
    RL_CUDA(ctx, rl::launch_gather(x, true, (const int*)(base + L.perm_pair), k, P, H, base + L.x_perm,
                                   w->gate_up_proj.qtype == RIALLM_COMPRESSION_FOUR_BIT, st),
            "gather");
    ctx->launches += 1;
  }
  if (int s = rl_ep_forward(ctx, w, x, out, T, H, I, E, k, flags, st, base, L, L.total)) return s;
  if (ctx->profiling) ctx->profiled_calls += 1;
  return RIALLM_OK;
}

int32_t riallm_cuda_moe_forward_ep_peer(riallm_ctx* ctx, const riallm_moe_weights* w, const void* x, void* out,
                                        int32_t T, int32_t H, int32_t I, int32_t E, int32_t k, uint32_t flags,
                                        void* stream) {
  if (!ctx || !w) return RIALLM_ERR_INVALID;
  if (!ctx->ep_peer) return set_err(ctx, RIALLM_ERR_CONFIG, "riallm_cuda_ep_peer_init was not called on this context");
  if (T < 1 || T > ctx->ep_peer_T || H != ctx->ep_peer_H || I != ctx->ep_peer_I || E != ctx->ep_peer_E ||
      k != ctx->ep_peer_k)
    return set_err(ctx, RIALLM_ERR_CONFIG, "call shape differs from riallm_cuda_ep_peer_init's (or T > its max_tokens)");
  if (!x || !out) return set_err(ctx, RIALLM_ERR_INVALID, "null x/out");
  if (int s = check_shapes(ctx, T, H, I, E, k)) return s;
  const int W = ctx->ep_world, EL = E / W;
  if (w->shared_gate_proj.data != nullptr)
    return set_err(ctx, RIALLM_ERR_CONFIG, "expert-parallel calls take routed experts only");
  if (int s = check_qtensor(ctx, w->gate, (uint64_t)E * H, "mlp.gate.weight", false)) return s;
  if (int s = check_qtensor(ctx, w->gate_up_proj, (uint64_t)EL * 2 * I * H, "mlp.experts.gate_up_proj", true))
    return s;
  if (int s = check_qtensor(ctx, w->down_proj, (uint64_t)EL * H * I, "mlp.experts.down_proj", true)) return s;
  if (!aligned16(x) || !aligned16(out)) return set_err(ctx, RIALLM_ERR_INVALID, "x/out must be 16-byte aligned");
  if (int s = set_device(ctx)) return s;
  const int P = T * k;
  MoeLayout L = rl::moe_layout(T, H, I, E, k, RIALLM_DTYPE_BF16, 0, ctx->num_sms);
  if (int s = ensure_arena(ctx, L.total)) return s;
  char* base = (char*)ctx->arena;
  cudaStream_t st = (cudaStream_t)stream;
  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_ROUTE);
    if (int s = route_into(ctx, w->gate, x, T, H, E, k, true, base, L, st)) return s;
    ctx->launches += 1;
  }
  {
    rl::PhaseTimer ps(ctx, st, RIALLM_PHASE_GATHER);
    RL_CUDA(ctx, rl::launch_gather(x, true, (const int*)(base + L.perm_pair), k, P, H, base + L.x_perm,
                                   w->gate_up_proj.qtype == RIALLM_COMPRESSION_FOUR_BIT, st),
            "gather");
    ctx->launches += 1;
  }
  if (int s = rl_ep_peer_forward(ctx, w, out, T, H, I, E, k, flags, st, base, L)) return s;
  if (ctx->profiling) ctx->profiled_calls += 1;
  return RIALLM_OK;
}

int32_t riallm_cuda_event_create(riallm_ctx* ctx, void** event_out) {
  if (!ctx || !event_out) return RIALLM_ERR_INVALID;
  if (int s = set_device(ctx)) return s;
  cudaEvent_t e = nullptr;
  RL_CUDA(ctx, cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
  *event_out = e;
  return RIALLM_OK;
}

int32_t riallm_cuda_event_destroy(riallm_ctx* ctx, void* event) {
  if (!ctx || !event) return RIALLM_ERR_INVALID;
  RL_CUDA(ctx, cudaEventDestroy((cudaEvent_t)event), "cudaEventDestroy");
  return RIALLM_OK;
}

int32_t riallm_cuda_event_record(riallm_ctx* ctx, void* event, void* stream) {
  if (!ctx || !event) return RIALLM_ERR_INVALID;
  RL_CUDA(ctx, cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream), "cudaEventRecord");
  return RIALLM_OK;
}

int32_t riallm_cuda_stream_wait_event(riallm_ctx* ctx, void* stream, void* event) {
  if (!ctx || !event) return RIALLM_ERR_INVALID;
  RL_CUDA(ctx, cudaStreamWaitEvent((cudaStream_t)stream, (cudaEvent_t)event, 0), "cudaStreamWaitEvent");
  return RIALLM_OK;
}

int32_t riallm_cuda_event_synchronize(riallm_ctx* ctx, void* event) {
  if (!ctx || !event) return RIALLM_ERR_INVALID;
  RL_CUDA(ctx, cudaEventSynchronize((cudaEvent_t)event), "cudaEventSynchronize");
  return RIALLM_OK;
}

int32_t riallm_cuda_ctx_set_wait_limit(riallm_ctx* ctx, uint64_t wait_ns) {
  if (!ctx) return RIALLM_ERR_INVALID;
  if (wait_ns != 0 && wait_ns < 1000)
    return set_err(ctx, RIALLM_ERR_CONFIG, "wait limit must be 0 (default) or at least 1000 ns");
  ctx->flag_wait_ns = wait_ns;
  return RIALLM_OK;
}

int32_t riallm_cuda_ctx_expire_next_wait(riallm_ctx* ctx) {
  if (!ctx) return RIALLM_ERR_INVALID;
  ctx->expire_next_wait = true;
  return RIALLM_OK;
}

int32_t riallm_cuda_profile_enable(riallm_ctx* ctx, int32_t enable) {
  if (!ctx) return RIALLM_ERR_INVALID;
  ctx->profiling = enable != 0;
  return RIALLM_OK;
}

int32_t riallm_cuda_profile_read(riallm_ctx* ctx, float* ms_per_phase, uint64_t* calls) {
  if (!ctx) return RIALLM_ERR_INVALID;
  float acc[RIALLM_NUM_PHASES] = {0};
  int status = RIALLM_OK;
  for (auto& pe : ctx->pending) {
    float ms = 0.0f;
    cudaError_t e = cudaEventSynchronize(pe.stop);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, pe.start, pe.stop);
    if (e != cudaSuccess && status == RIALLM_OK) status = cuda_err(ctx, e, "profile event");
    if (pe.phase >= 0 && pe.phase < RIALLM_NUM_PHASES) acc[pe.phase] += ms;
    ctx->event_pool.push_back(pe.start);
    ctx->event_pool.push_back(pe.stop);
  }
  ctx->pending.clear();
  if (ms_per_phase)
    for (int i = 0; i < RIALLM_NUM_PHASES; ++i) ms_per_phase[i] = acc[i];
  if (calls) *calls = ctx->profiled_calls;
  ctx->profiled_calls = 0;
  return status;
}

uint64_t riallm_cuda_launch_count(const riallm_ctx* ctx) { return ctx ? ctx->launches : 0; }

}  // extern "C"
