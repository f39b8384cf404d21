// decoder.cu -- the dense parts of a Mixtral-style decoder layer that sit
// around the MoE block, kept on the device with a bf16 KV cache:
//   * RMSNorm (src/model.rs:456-468) with an optional fused residual add;
//   * rotate-half rotary embedding (inv_freq = theta^(-2i/d),
//     src/model.rs:1002-1071) of q and k, with k and v appended to the cache;
//   * causal grouped-query attention over the cache (src/model.rs:912-1000,
//     the query heads of one KV head sharing it as repeat_heads does,
//     src/model.rs:1317-1328).
// All arithmetic is float32 with bf16 inputs and outputs. Positions come from
// a device array (one entry per sequence), so a decode step can be replayed
// from a CUDA graph.
#include <cfloat>

#include "common.cuh"
#include "internal.h"

namespace {

__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

constexpr int kNormThreads = 256;

// One CTA per row; H % 8 == 0 and rows 16-byte aligned (8 bf16 per load).
// With delta: x = bf16(x + delta) is stored back before the norm.
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_kernel(uint16_t* __restrict__ x, const uint16_t* __restrict__ delta,
                   const float* __restrict__ w, uint16_t* __restrict__ out, int H, float eps) {
  rl::pdl_wait();
  rl::pdl_launch_dependents();
  const size_t r = blockIdx.x;
  uint4* xr = reinterpret_cast<uint4*>(x + r * H);
  const uint4* dr = delta ? reinterpret_cast<const uint4*>(delta + r * H) : nullptr;
  const int nv = H / 8;
  float ss = 0.f;
  for (int v = threadIdx.x; v < nv; v += kNormThreads) {
    uint4 a = xr[v];
    uint16_t* ah = reinterpret_cast<uint16_t*>(&a);
    if (dr) {
      uint4 b = dr[v];
      const uint16_t* bh = reinterpret_cast<const uint16_t*>(&b);
#pragma unroll
      for (int j = 0; j < 8; ++j) ah[j] = f2bf(__fadd_rn(bf2f(ah[j]), bf2f(bh[j])));
      xr[v] = a;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = bf2f(ah[j]);
      ss = fmaf(f, f, ss);
    }
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)H), eps));
  uint4* orow = reinterpret_cast<uint4*>(out + r * H);
  for (int v = threadIdx.x; v < nv; v += kNormThreads) {
    uint4 a = xr[v];  // this thread's own stores above, if any
    const uint16_t* ah = reinterpret_cast<const uint16_t*>(&a);
    uint4 o;
    uint16_t* oh = reinterpret_cast<uint16_t*>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) oh[j] = f2bf(__fmul_rn(__fmul_rn(bf2f(ah[j]), inv), w[v * 8 + j]));
    orow[v] = o;
  }
}

// CTA (row, head group): row b*T + t of qkv [B*T, (nh + 2 nkv) * d] (q heads,
// then k heads, then v heads) sits at position pos[b] + t. Head group g
// covers heads [8g, 8g + 8): q and k heads are rotated (q to q_out, k into
// the cache), v heads copied into the cache. Positions outside [0, S_max)
// write nothing to the caches (the attention kernel clamps the same way).
constexpr int kRopeHeads = 8;
__global__ void __launch_bounds__(128)
    rope_append_kernel(const uint16_t* __restrict__ qkv, const int* __restrict__ pos, int T, int nh,
                       int nkv, int d, const float* __restrict__ inv_freq,
                       uint16_t* __restrict__ q_out, uint16_t* __restrict__ kc,
                       uint16_t* __restrict__ vc, int S_max) {
  __shared__ float cs[rl::kAttnMaxD / 2], sn[rl::kAttnMaxD / 2];
  rl::pdl_wait();
  rl::pdl_launch_dependents();
  const int row = blockIdx.x;
  const int b = row / T, t = row - b * T;
  const int p = pos[b] + t;
  const bool in_cache = p >= 0 && p < S_max;
  const int half = d >> 1;
  const int h0 = blockIdx.y * kRopeHeads;
  const int h1 = min(h0 + kRopeHeads, nh + 2 * nkv);
  const uint16_t* src = qkv + (size_t)row * (nh + 2 * nkv) * d;
  if (h0 < nh + nkv) {
    for (int j = threadIdx.x; j < half; j += blockDim.x) {
      float s_, c_;
      sincosf(__fmul_rn((float)p, inv_freq[j]), &s_, &c_);
      cs[j] = c_;
      sn[j] = s_;
    }
    __syncthreads();
  }
  const int hr = min(h1, nh + nkv);  // rotated heads of this group: [h0, hr)
  for (int i = threadIdx.x; i < (hr - h0) * half; i += blockDim.x) {
    const int h = h0 + i / half, j = i % half;
    const float c = cs[j], s = sn[j];
    const float x1 = bf2f(src[h * d + j]), x2 = bf2f(src[h * d + j + half]);
    const uint16_t o1 = f2bf(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
    const uint16_t o2 = f2bf(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
    if (h < nh) {
      uint16_t* q = q_out + (size_t)row * nh * d + (size_t)h * d;
      q[j] = o1;
      q[j + half] = o2;
    } else if (in_cache) {
      uint16_t* k = kc + (((size_t)b * nkv + (h - nh)) * S_max + p) * d;
      k[j] = o1;
      k[j + half] = o2;
    }
  }
  const int v0 = max(h0, nh + nkv);  // copied v heads: [v0, h1)
  if (in_cache && v0 < h1) {
    for (int i = threadIdx.x; i < (h1 - v0) * d; i += blockDim.x) {
      const int h = v0 + i / d, j = i % d;
      vc[(((size_t)b * nkv + (h - nh - nkv)) * S_max + p) * d + j] = src[(size_t)h * d + j];
    }
  }
}

// Skinny bf16 linear layer y = x · wᵀ for decode batches (M <= 8 rows of
// x): the weight [N, K] is streamed once. Each warp takes whole output
// columns n (rows of w): lane l reads 16-byte pieces l, l + 32, ... of w[n]
// and the same pieces of every x row (L1-resident after the first warp),
// accumulates M float32 dot products and the warp reduces them in a fixed
// butterfly. K % 256 == 0.
template <int M>
__global__ void __launch_bounds__(256)
    linear_bf16_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                       uint16_t* __restrict__ y, int N, int K) {
  rl::pdl_wait();
  rl::pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int kv = K >> 3;  // 16-byte pieces per row
  for (int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < N; n += warps) {
    const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)n * K);
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.f;
#pragma unroll 4
    for (int v = lane; v < kv; v += 32) {
      const uint4 wv = __ldcs(wr + v);  // streamed once: evict first
      const uint16_t* wh = reinterpret_cast<const uint16_t*>(&wv);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * K) + v);
        const uint16_t* xh = reinterpret_cast<const uint16_t*>(&xv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[m] = fmaf(bf2f(xh[e]), bf2f(wh[e]), acc[m]);
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float a = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) y[(size_t)m * N + n] = f2bf(a);
    }
  }
}

constexpr int kKeyChunk = 64;

// CTA (t * nsplit + split, kv head, b), D threads (one per head dimension):
// the REP query heads of KV head kh for token t of sequence b attend keys
// [0, L), L = pos[b] + t + 1; split s takes the s-th of nsplit equal
// contiguous key ranges. Keys are taken kKeyChunk at a time: scores (a
// thread per key), the chunk's max and exp-sum per head, then the weighted
// values (a thread per dimension), rescaling the running sums online. With
// nsplit > 1 each CTA stores its maxima, sums and accumulators in ws and the
// group's last CTA (a counter per group) merges them in split order.
template <int D, int REP>
__global__ void __launch_bounds__(D)
    attention_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ kc,
                     const uint16_t* __restrict__ vc, const int* __restrict__ pos, int T, int nh,
                     int nkv, int S_max, float scale, int nsplit, float* __restrict__ ws,
                     unsigned* __restrict__ counters, uint16_t* __restrict__ out) {
  constexpr int NW = D / 32;
  rl::pdl_wait();
  rl::pdl_launch_dependents();
  const int split = blockIdx.x % nsplit, t = blockIdx.x / nsplit;
  const int kh = blockIdx.y, b = blockIdx.z;
  const int i = threadIdx.x, lane = i & 31, warp = i >> 5;
  const size_t row = (size_t)b * T + t;
  int L = pos[b] + t + 1;
  L = L < 0 ? 0 : (L > S_max ? S_max : L);
  const int per = (L + nsplit - 1) / nsplit;
  const int k0 = min(L, split * per), k1 = min(L, k0 + per);
  __shared__ float qs[REP][D];
  __shared__ float ps[REP][kKeyChunk];
  // The chunk's key and value rows, staged with cp.async; key rows keep
  // their 16-byte pieces XOR-swizzled by the row so that a thread per key
  // reads them without bank conflicts.
  __shared__ __align__(16) uint16_t ks[kKeyChunk][D];
  __shared__ __align__(16) uint16_t vs[kKeyChunk][D];
  __shared__ float red[REP][NW];
  __shared__ float bc[REP];
  __shared__ unsigned last;
#pragma unroll
  for (int r = 0; r < REP; ++r) qs[r][i] = bf2f(q[row * nh * D + (size_t)(kh * REP + r) * D + i]);
  __syncthreads();
  const size_t base = ((size_t)b * nkv + kh) * S_max * D;
  const uint16_t* kb = kc + base;
  const uint16_t* vb = vc + base;
  float acc[REP], m[REP], l[REP];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    acc[r] = 0.f;
    m[r] = -FLT_MAX;
    l[r] = 0.f;
  }
  for (int c0 = k0; c0 < k1; c0 += kKeyChunk) {
    const int n = min(kKeyChunk, k1 - c0);
    float cmax[REP];
#pragma unroll
    for (int r = 0; r < REP; ++r) cmax[r] = -FLT_MAX;
    constexpr int kPieces = D / 8;  // 16-byte pieces per row
    for (int idx = i; idx < n * kPieces; idx += D) {
      const int j = idx / kPieces, v = idx - j * kPieces;
      rl::cp_async_16(&ks[j][(v ^ (j & 7)) * 8], kb + (size_t)(c0 + j) * D + v * 8);
      rl::cp_async_16(&vs[j][v * 8], vb + (size_t)(c0 + j) * D + v * 8);
    }
    rl::cp_async_commit();
    rl::cp_async_wait<0>();
    __syncthreads();
    for (int j = i; j < n; j += D) {
      float s[REP];
#pragma unroll
      for (int r = 0; r < REP; ++r) s[r] = 0.f;
#pragma unroll 4
      for (int v = 0; v < D / 8; ++v) {
        uint4 kv = *reinterpret_cast<const uint4*>(&ks[j][(v ^ (j & 7)) * 8]);
        const uint16_t* kh16 = reinterpret_cast<const uint16_t*>(&kv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float kf = bf2f(kh16[e]);
#pragma unroll
          for (int r = 0; r < REP; ++r) s[r] = fmaf(qs[r][v * 8 + e], kf, s[r]);
        }
      }
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        const float sc = __fmul_rn(s[r], scale);
        ps[r][j] = sc;
        cmax[r] = fmaxf(cmax[r], sc);
      }
    }
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      float v = cmax[r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) red[r][warp] = v;
    }
    __syncthreads();
    float mn[REP], corr[REP];
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      float v = red[r][0];
#pragma unroll
      for (int w = 1; w < NW; ++w) v = fmaxf(v, red[r][w]);
      mn[r] = fmaxf(m[r], v);
      corr[r] = expf(m[r] - mn[r]);
      m[r] = mn[r];
    }
    __syncthreads();  // red is reused below
    float csum[REP];
#pragma unroll
    for (int r = 0; r < REP; ++r) csum[r] = 0.f;
    for (int j = i; j < n; j += D) {
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        const float e = expf(ps[r][j] - mn[r]);
        ps[r][j] = e;
        csum[r] += e;
      }
    }
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      float v = csum[r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[r][warp] = v;
    }
    __syncthreads();
    if (i < REP) {
      float v = 0.f;
      for (int w = 0; w < NW; ++w) v += red[i][w];
      bc[i] = v;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      l[r] = fmaf(l[r], corr[r], bc[r]);
      acc[r] *= corr[r];
    }
#pragma unroll 8
    for (int j = 0; j < n; ++j) {
      const float vv = bf2f(vs[j][i]);
#pragma unroll
      for (int r = 0; r < REP; ++r) acc[r] = fmaf(ps[r][j], vv, acc[r]);
    }
    __syncthreads();  // ps and red are rewritten by the next chunk
  }
  uint16_t* orow = out + row * nh * D + (size_t)kh * REP * D + i;
  if (nsplit == 1) {
#pragma unroll
    for (int r = 0; r < REP; ++r) orow[(size_t)r * D] = f2bf(L > 0 ? __fdiv_rn(acc[r], l[r]) : 0.f);
    return;
  }
  // Partial of this split: [m x REP][l x REP][acc REP x D].
  constexpr int kSlot = REP * (D + 2);
  const size_t group = ((size_t)b * nkv + kh) * T + t;
  float* slot = ws + (group * nsplit + split) * kSlot;
  if (i == 0) {
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      slot[r] = m[r];
      slot[REP + r] = l[r];
    }
  }
#pragma unroll
  for (int r = 0; r < REP; ++r) slot[2 * REP + r * D + i] = acc[r];
  __threadfence();
  __syncthreads();
  if (i == 0) last = atomicAdd(counters + group, 1u) == (unsigned)(nsplit - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  // Merge: the splits' maxima and sums are staged in shared memory (ps is
  // free now; nsplit <= 32), thread r < REP turns them into weights
  // exp(m_s - M) and the denominator, then every thread sums its dimension
  // over the splits in split order.
  const float* g0 = ws + group * nsplit * kSlot;
  for (int x = i; x < REP * nsplit; x += D) {
    const int r = x / nsplit, sp = x - r * nsplit;
    ps[r][sp] = __ldcg(g0 + sp * kSlot + r);
    ps[r][32 + sp] = __ldcg(g0 + sp * kSlot + REP + r);
  }
  __syncthreads();
  if (i < REP) {
    float M = -FLT_MAX;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, ps[i][sp]);
    float den = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float w = expf(ps[i][sp] - M);
      ps[i][sp] = w;
      den = fmaf(w, ps[i][32 + sp], den);
    }
    bc[i] = den;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float num = 0.f;
#pragma unroll 8
    for (int sp = 0; sp < nsplit; ++sp) num = fmaf(ps[r][sp], __ldcg(g0 + sp * kSlot + 2 * REP + r * D + i), num);
    orow[(size_t)r * D] = f2bf(L > 0 ? __fdiv_rn(num, bc[r]) : 0.f);
  }
  if (i == 0) counters[group] = 0u;  // ready for the next call
}

template <int D>
cudaError_t launch_attention_d(int rep, dim3 grid, const uint16_t* q, const uint16_t* kc,
                               const uint16_t* vc, const int* pos, int T, int nh, int nkv,
                               int S_max, float scale, int nsplit, float* ws, unsigned* counters,
                               uint16_t* out, cudaStream_t st) {
  switch (rep) {
#define RL_ATTN_CASE(R)                                                                       \
  case R:                                                                                     \
    return rl::launch_pdl(attention_kernel<D, R>, grid, dim3(D), 0, st, q, kc, vc, pos, T, nh, nkv, S_max, \
                      scale, nsplit, ws, counters, out);
    RL_ATTN_CASE(1)
    RL_ATTN_CASE(2)
    RL_ATTN_CASE(4)
    RL_ATTN_CASE(6)
    RL_ATTN_CASE(8)
#undef RL_ATTN_CASE
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int fail(riallm_ctx* ctx, int code, const char* msg) {
  ctx->last_error = msg;
  return code;
}

int launch_status(riallm_ctx* ctx, cudaError_t e, const char* what) {
  if (e == cudaSuccess) {
    ctx->launches += 1;
    return RIALLM_OK;
  }
  ctx->last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return RIALLM_ERR_CUDA;
}

}  // namespace

extern "C" {

int32_t riallm_cuda_rmsnorm(riallm_ctx* ctx, void* x, const void* delta, const float* w, void* out,
                            int32_t rows, int32_t H, float eps, void* stream) {
  if (!ctx || !x || !w || !out) return RIALLM_ERR_INVALID;
  if (rows < 0 || H <= 0 || H % 8 != 0) return fail(ctx, RIALLM_ERR_CONFIG, "rmsnorm: need H % 8 == 0");
  if (!al16(x) || !al16(out) || (delta && !al16(delta)))
    return fail(ctx, RIALLM_ERR_INVALID, "rmsnorm: buffers must be 16-byte aligned");
  if (rows == 0) return RIALLM_OK;
  if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, RIALLM_ERR_CUDA, "cudaSetDevice");
  cudaError_t e = rl::launch_pdl(rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0, (cudaStream_t)stream,
                             static_cast<uint16_t*>(x), static_cast<const uint16_t*>(delta), w,
                             static_cast<uint16_t*>(out), H, eps);
  return launch_status(ctx, e, "rmsnorm launch");
}

int32_t riallm_cuda_rope_kv_append(riallm_ctx* ctx, const void* qkv, const int32_t* pos, int32_t B,
                                   int32_t T, int32_t nh, int32_t nkv, int32_t d,
                                   const float* inv_freq, void* q_out, void* k_cache,
                                   void* v_cache, int32_t S_max, void* stream) {
  if (!ctx || !qkv || !pos || !inv_freq || !q_out || !k_cache || !v_cache) return RIALLM_ERR_INVALID;
  if (B < 0 || T < 0 || nh <= 0 || nkv <= 0 || d <= 0 || (d & 1) || d > rl::kAttnMaxD || S_max <= 0)
    return fail(ctx, RIALLM_ERR_CONFIG, "rope_kv_append: bad dimensions (head_dim even, <= 128)");
  if ((int64_t)nh + 2 * nkv > 65535 * kRopeHeads) return fail(ctx, RIALLM_ERR_CONFIG, "rope_kv_append: too many heads");
  if ((int64_t)B * T == 0) return RIALLM_OK;
  if ((int64_t)B * T > (1ll << 31) - 1) return fail(ctx, RIALLM_ERR_CONFIG, "rope_kv_append: too many rows");
  if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, RIALLM_ERR_CUDA, "cudaSetDevice");
  const dim3 grid(B * T, (nh + 2 * nkv + kRopeHeads - 1) / kRopeHeads);
  cudaError_t e = rl::launch_pdl(rope_append_kernel, grid, dim3(128), 0, (cudaStream_t)stream,
                             static_cast<const uint16_t*>(qkv), pos, T, nh, nkv, d, inv_freq,
                             static_cast<uint16_t*>(q_out), static_cast<uint16_t*>(k_cache),
                             static_cast<uint16_t*>(v_cache), S_max);
  return launch_status(ctx, e, "rope_kv_append launch");
}

int32_t riallm_cuda_attention(riallm_ctx* ctx, const void* q, const void* k_cache, const void* v_cache,
                              const int32_t* pos, int32_t B, int32_t T, int32_t nh, int32_t nkv,
                              int32_t d, int32_t S_max, void* out, void* stream) {
  if (!ctx || !q || !k_cache || !v_cache || !pos || !out) return RIALLM_ERR_INVALID;
  if (B < 0 || T < 0 || nh <= 0 || nkv <= 0 || S_max <= 0 || nh % nkv != 0)
    return fail(ctx, RIALLM_ERR_CONFIG, "attention: bad dimensions (heads must be a multiple of kv heads)");
  const int rep = nh / nkv;
  if (d != 64 && d != 128) return fail(ctx, RIALLM_ERR_CONFIG, "attention: head_dim must be 64 or 128");
  if (rep != 1 && rep != 2 && rep != 4 && rep != 6 && rep != 8)
    return fail(ctx, RIALLM_ERR_CONFIG, "attention: heads / kv heads must be 1, 2, 4, 6 or 8");
  if (!al16(k_cache) || !al16(v_cache))
    return fail(ctx, RIALLM_ERR_INVALID, "attention: k and v caches must be 16-byte aligned");
  if (B > 65535 || nkv > 65535) return fail(ctx, RIALLM_ERR_CONFIG, "attention: batch or kv heads too large");
  if ((int64_t)B * T == 0) return RIALLM_OK;
  if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, RIALLM_ERR_CUDA, "cudaSetDevice");
  // Split each (sequence, kv head, token) group's keys over several CTAs when
  // the groups alone would leave SMs idle (decode at small batch).
  const int64_t groups = (int64_t)B * T * nkv;
  int nsplit = 1;
  if (groups < 2ll * ctx->num_sms) {
    nsplit = (int)((2ll * ctx->num_sms + groups - 1) / groups);
    nsplit = min(nsplit, (int)(4ll * ctx->num_sms / groups));
    nsplit = min(nsplit, 32);
    nsplit = max(1, min(nsplit, S_max / 64));  // at least 64 keys per split at full length
  }
  if ((int64_t)T * nsplit > 0x7fffffffll) return fail(ctx, RIALLM_ERR_CONFIG, "attention: too many tokens");
  const dim3 grid(T * nsplit, nkv, B);
  const float scale = (float)(1.0 / sqrt((double)d));
  auto* qq = static_cast<const uint16_t*>(q);
  auto* kk = static_cast<const uint16_t*>(k_cache);
  auto* vv = static_cast<const uint16_t*>(v_cache);
  auto* oo = static_cast<uint16_t*>(out);
  auto* counters = static_cast<unsigned*>(ctx->attn_ws);
  float* ws = reinterpret_cast<float*>(static_cast<char*>(ctx->attn_ws) + rl::kAttnCounterBytes);
  cudaError_t e = d == 128 ? launch_attention_d<128>(rep, grid, qq, kk, vv, pos, T, nh, nkv, S_max, scale, nsplit,
                                                     ws, counters, oo, (cudaStream_t)stream)
                           : launch_attention_d<64>(rep, grid, qq, kk, vv, pos, T, nh, nkv, S_max, scale, nsplit,
                                                    ws, counters, oo, (cudaStream_t)stream);
  return launch_status(ctx, e, "attention launch");
}

int32_t riallm_cuda_linear_bf16(riallm_ctx* ctx, const void* x, const void* w, void* y, int32_t M,
                                int32_t N, int32_t K, void* stream) {
  if (!ctx || !x || !w || !y) return RIALLM_ERR_INVALID;
  if (M < 0 || N < 0 || K <= 0 || M > 8 || K % 256 != 0)
    return fail(ctx, RIALLM_ERR_CONFIG, "linear_bf16: need M <= 8 and K % 256 == 0");
  if (!al16(x) || !al16(w)) return fail(ctx, RIALLM_ERR_INVALID, "linear_bf16: x and w must be 16-byte aligned");
  if (M == 0 || N == 0) return RIALLM_OK;
  if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, RIALLM_ERR_CUDA, "cudaSetDevice");
  const int warps_needed = N;
  int blocks = (warps_needed + 7) / 8;
  const int cap = ctx->num_sms * 8;  // 8 CTAs of 8 warps per SM at most
  if (blocks > cap) blocks = cap;
  auto* xx = static_cast<const uint16_t*>(x);
  auto* ww = static_cast<const uint16_t*>(w);
  auto* yy = static_cast<uint16_t*>(y);
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e;
  switch (M) {
#define RL_LIN_CASE(R) \
  case R:              \
    e = rl::launch_pdl(linear_bf16_kernel<R>, dim3(blocks), dim3(256), 0, st, xx, ww, yy, N, K); \
    break;
    RL_LIN_CASE(1)
    RL_LIN_CASE(2)
    RL_LIN_CASE(3)
    RL_LIN_CASE(4)
    RL_LIN_CASE(5)
    RL_LIN_CASE(6)
    RL_LIN_CASE(7)
    RL_LIN_CASE(8)
#undef RL_LIN_CASE
    default:
      e = cudaErrorInvalidValue;
  }
  return launch_status(ctx, e, "linear_bf16 launch");
}

}  // extern "C"
