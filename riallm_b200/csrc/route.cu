// route.cu -- router, token permutation, gather, combine, and the CUDA-core
// grouped GEMM used by the float32 path and the shared expert.
//
// Router arithmetic is fixed so routing is reproducible bit for bit:
//   logit[t,e] = xor-butterfly sum (offsets 16,8,4,2,1) of 32 lane partials;
//     lane l accumulates, with fused multiply-adds, the 8-element chunks
//     c = l, l+32, ... of x[t] . wg[e] in ascending order;
//   softmax: max, own exp (Cody-Waite + degree-7 Taylor, fused), sequential
//     sum over e, IEEE division;
//   top-k: stable descending order (ties to the lower expert index), as
//     candle's arg_sort_last_dim(false) in src/model.rs:764-767;
//   renormalise by the sequential sum of the k picked probabilities
//     (src/model.rs:768-770).
#include "common.cuh"
#include "internal.h"

namespace rl {

constexpr unsigned kFull = 0xffffffffu;

// e^x: Cody & Waite argument reduction x = n ln2 + r with ln2 split into a
// 16-bit head and a tail, degree-7 Taylor polynomial of e^r (|r| <= ln2/2,
// truncation < 6e-9 relative) in fused Horner form, times 2^n. Inputs below
// -87 return 0; the router only feeds x - max <= 0.
__device__ __forceinline__ float own_expf(float x) {
  if (x != x) return x;
  if (x < -87.0f) return 0.0f;
  if (x > 88.0f) return __int_as_float(0x7f800000);
  const float t = __fmul_rn(x, 0x1.715476p+0f);
  const float n = rintf(t);
  float r = __fmaf_rn(-n, 0x1.62e4p-1f, x);
  r = __fmaf_rn(-n, 0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
  p = __fmaf_rn(p, r, 0x1.111112p-7f);
  p = __fmaf_rn(p, r, 0x1.555556p-5f);
  p = __fmaf_rn(p, r, 0x1.555556p-3f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = (int)n;
  const float scale = __int_as_float((ni + 127) << 23);
  return __fmul_rn(p, scale);
}

__device__ __forceinline__ void load_chunk8(const void* x, bool x_bf16, uint64_t off, float (&v)[8]) {
  if (x_bf16) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + off));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + off);
    float4 a = __ldg(p), b = __ldg(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// One warp per token. Shared memory: per warp E logits and E probabilities.
// Eight consecutive elements g0..g0+7 (g0 a multiple of 8) of the router
// weight as float32, decoded like QuantizedTensor::dequantize
// (src/quantization.rs:45-95): value = (code - zero) * scale. NF4 element e
// reads nibble e%2 of byte e/2 and block (e+1)/64, so only element 7 of a
// chunk can sit in the next block; 8-bit element e reads block e/128. A
// block past the parameter arrays uses scale 1.0 / zero 0.0.
template <int QT>
__device__ __forceinline__ void gate_chunk8(const RouterArgs& a, uint64_t g0, float (&w)[8]) {
  if (QT == RIALLM_COMPRESSION_NONE) {
    const float* src = reinterpret_cast<const float*>(a.gdata) + g0;
    if (a.gate_v8) {
      // One 256-bit load per lane: two 128-bit loads 32 bytes apart would
      // fetch every 32-byte sector of a warp's 1 KiB twice through L1.
      // Not volatile, so the compiler may schedule it early within the
      // chunk loops; those loops start after pdl_wait() and the staging
      // barrier, and the weight is not written while the kernel runs.
      asm("ld.global.nc.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                   : "=f"(w[0]), "=f"(w[1]), "=f"(w[2]), "=f"(w[3]), "=f"(w[4]), "=f"(w[5]), "=f"(w[6]), "=f"(w[7])
                   : "l"(src));
    } else {
      const float4* p = reinterpret_cast<const float4*>(src);
      const float4 u = __ldg(p), v = __ldg(p + 1);
      w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
      w[4] = v.x; w[5] = v.y; w[6] = v.z; w[7] = v.w;
    }
  } else if (QT == RIALLM_COMPRESSION_FOUR_BIT) {
    const uint32_t codes = __ldg(reinterpret_cast<const uint32_t*>(a.gdata) + g0 / 8);
    const uint64_t b0 = g0 >> 6, b7 = (g0 + 8) >> 6;
    const float s0 = b0 < a.n_scales ? __ldg(a.gscales + b0) : 1.0f;
    const float z0 = b0 < a.n_zeros ? __ldg(a.gzeros + b0) : 0.0f;
    const float s7 = b7 < a.n_scales ? __ldg(a.gscales + b7) : 1.0f;
    const float z7 = b7 < a.n_zeros ? __ldg(a.gzeros + b7) : 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float code = (float)((codes >> (4 * i)) & 15u);
      w[i] = i == 7 ? __fmul_rn(__fsub_rn(code, z7), s7) : __fmul_rn(__fsub_rn(code, z0), s0);
    }
  } else {
    const uint2 codes = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(a.gdata) + g0));
    const uint64_t b = g0 >> 7;
    const float s = b < a.n_scales ? __ldg(a.gscales + b) : 1.0f;
    const float z = b < a.n_zeros ? __ldg(a.gzeros + b) : 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t word = i < 4 ? codes.x : codes.y;
      const float code = (float)((word >> (8 * (i & 3))) & 255u);
      w[i] = __fmul_rn(__fsub_rn(code, z), s);
    }
  }
}

// Stable counting sort of the P (token, choice) pairs by expert, run by one
// CTA of kRouterThreads threads: per-warp histograms over contiguous pair
// segments, an exclusive scan per expert, then each warp walks its segment
// in order and ranks equal experts inside every 32-pair batch with
// match_any, so each expert's pairs keep pair order.
__device__ void permute_block(const int* topk_idx, int P, int E, int* counts, int* offsets,
                              int* perm_pair, int* inv_pos, int* hist, int* off_s) {
  constexpr int W = kRouterThreads / 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int stride = E + 1;
  for (int i = tid; i < W * stride; i += kRouterThreads) hist[i] = 0;
  __syncthreads();
  const int per = (P + W - 1) / W;
  const int p0 = min(P, warp * per), p1 = min(P, p0 + per);
  for (int p = p0 + lane; p < p1; p += 32) atomicAdd(&hist[warp * stride + __ldcg(topk_idx + p)], 1);
  __syncthreads();
  for (int e = tid; e < E; e += kRouterThreads) {
    int c = 0;
    for (int w = 0; w < W; ++w) c += hist[w * stride + e];
    off_s[e + 1] = c;
  }
  __syncthreads();
  if (tid == 0) {
    off_s[0] = 0;
    for (int e = 0; e < E; ++e) off_s[e + 1] += off_s[e];
  }
  __syncthreads();
  for (int e = tid; e < E; e += kRouterThreads) {
    int b = off_s[e];
    counts[e] = off_s[e + 1] - off_s[e];
    for (int w = 0; w < W; ++w) {
      const int h = hist[w * stride + e];
      hist[w * stride + e] = b;
      b += h;
    }
  }
  for (int e = tid; e <= E; e += kRouterThreads) offsets[e] = off_s[e];
  __syncthreads();
  for (int base = p0; base < p1; base += 32) {
    const int p = base + lane;
    const bool valid = p < p1;
    const unsigned act = __ballot_sync(kFull, valid);
    if (valid) {
      const int e = __ldcg(topk_idx + p);
      const unsigned peers = __match_any_sync(act, e);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      const int pos = hist[warp * stride + e] + rank;
      perm_pair[pos] = p;
      if (inv_pos) inv_pos[p] = pos;
      __syncwarp(act);
      if (rank == 0) hist[warp * stride + e] += __popc(peers);
    }
    __syncwarp();
  }
}

// Bulk L2 prefetch of this CTA's 1/gridDim share of [base, base + bytes),
// trimmed to 16-byte boundaries inside the buffer.
__device__ __forceinline__ void prefetch_share(const void* base, uint64_t bytes) {
  if (!base || bytes == 0) return;
  const uint64_t b = reinterpret_cast<uint64_t>(base), e = b + bytes;
  const uint64_t per = (bytes + gridDim.x - 1) / gridDim.x;
  uint64_t lo = b + per * blockIdx.x, hi = lo + per;
  if (hi > e) hi = e;
  lo = (lo + 15) & ~uint64_t(15);
  hi &= ~uint64_t(15);
  while (lo < hi) {
    const uint64_t n = hi - lo < (1u << 20) ? hi - lo : (1u << 20);
    bulk_prefetch_l2(reinterpret_cast<const void*>(lo), (uint32_t)n);
    lo += n;
  }
}

// A CTA routes TT consecutive tokens: warp w computes the logits of experts
// w, w+8, ... for all of them, decoding each 8-element chunk of the router
// weight once and applying it to the TT staged token rows (each token's
// fused multiply-add chain runs in exactly the per-token order above); warp
// t (t < TT) then takes token t's softmax and top k. TT = 1 for decode-sized
// calls (one CTA per token), 4 or 8 for prefills, where the router weight
// would otherwise be decoded once per token. Pair sorting: for up to
// kSortOneCta pairs the CTA that finishes last (a counter in device memory,
// zero between calls and reset by that CTA) sorts all pairs by expert;
// above it every CTA counts its own pairs per expert, the last CTA turns
// those counts into per-CTA bases (scatter_kernel places the pairs).
// EB experts per warp pass: each staged x chunk is read from shared memory
// once for EB experts (with EB = 1 the shared-memory reads of x, one per
// FMA group, bound the kernel). Every (token, expert) logit still sums its
// chunks and elements in the same order.
template <int QT, int TT, int EB>
__global__ void __launch_bounds__(kRouterThreads) router_kernel(const RouterArgs a) {
  static_assert(TT == 1 || TT % 2 == 0, "token tiles of 1 or of whole token pairs");
  extern __shared__ float sm[];
  __shared__ int is_last;
  // The router weight does not depend on the previous kernel: while it
  // drains, pull this CTA's share of it into L2 (the loads below then hit L2).
  if (threadIdx.x == 0) {
    const uint64_t wbytes = QT == RIALLM_COMPRESSION_FOUR_BIT ? (uint64_t)a.E * a.H / 2
                            : QT == RIALLM_COMPRESSION_EIGHT_BIT ? (uint64_t)a.E * a.H
                                                                 : (uint64_t)a.E * a.H * 4;
    prefetch_share(a.gdata, wbytes);
    if (QT != RIALLM_COMPRESSION_NONE) {
      prefetch_share(a.gscales, a.n_scales * 4);
      prefetch_share(a.gzeros, a.n_zeros * 4);
    }
  }
  pdl_wait();  // x comes from the previous kernel; every output is read by earlier ones
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.E, H = a.H, k = a.k;
  const int t0 = blockIdx.x * TT;
  const int nt = min(TT, a.T - t0);
  float* lg = sm;             // [TT][E] logits (then "taken" marks)
  float* pr = sm + TT * E;    // [TT][E] probabilities
  int* hist = reinterpret_cast<int*>(sm + 2 * TT * E);
  int* off_s = hist + (kRouterThreads / 32) * (E + 1);
  // The tile's token rows as float32, staged once (16-byte aligned).
  float* xs = sm + ((2 * TT * E + (kRouterThreads / 32) * (E + 1) + E + 1 + 3) & ~3);
  const int nchunk = H >> 3;
  if constexpr (TT == 1) {
    for (int i = threadIdx.x; i < TT * nchunk; i += kRouterThreads) {
      const int t = i / nchunk, c = i - t * nchunk;
      float xv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (t < nt) load_chunk8(a.x, a.x_bf16 != 0, (uint64_t)(t0 + t) * H + 8ull * c, xv);
      // The row is stored as the first halves of all its chunks, then the
      // second halves, so the 32 lanes' 16-byte reads of one half are 512
      // contiguous bytes (no bank conflicts).
      float* d = xs + (uint64_t)t * H + 4 * c;
      *reinterpret_cast<float4*>(d) = make_float4(xv[0], xv[1], xv[2], xv[3]);
      *reinterpret_cast<float4*>(d + 4 * nchunk) = make_float4(xv[4], xv[5], xv[6], xv[7]);
    }
  } else {
    // Tokens 2u and 2u+1 interleaved: the float4 at xs + ((4u + q) nchunk + c) 4
    // holds elements 8c+2q and 8c+2q+1 of both, as {x[2u][8c+2q],
    // x[2u+1][8c+2q], x[2u][8c+2q+1], x[2u+1][8c+2q+1]}, so one read gives
    // two (token 2u, token 2u+1) operand pairs of the packed FMAs below, and
    // the 32 lanes' reads of one (u, q) are 512 contiguous bytes. A token
    // past the tile's end is staged as zeros (its logits are not used).
    for (int i = threadIdx.x; i < (TT / 2) * nchunk; i += kRouterThreads) {
      const int u = i / nchunk, c = i - u * nchunk;
      float xa[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      float xb[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (2 * u < nt) load_chunk8(a.x, a.x_bf16 != 0, (uint64_t)(t0 + 2 * u) * H + 8ull * c, xa);
      if (2 * u + 1 < nt) load_chunk8(a.x, a.x_bf16 != 0, (uint64_t)(t0 + 2 * u + 1) * H + 8ull * c, xb);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<float4*>(xs + ((uint64_t)(4 * u + q) * nchunk + c) * 4) =
            make_float4(xa[2 * q], xb[2 * q], xa[2 * q + 1], xb[2 * q + 1]);
    }
  }
  __syncthreads();
  for (int e0 = warp * EB; e0 < E; e0 += (kRouterThreads / 32) * EB) {
    float acc[TT][EB];
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
      for (int j = 0; j < EB; ++j) acc[t][j] = 0.0f;
    if constexpr (TT == 1 && QT == RIALLM_COMPRESSION_NONE) {
      // One token per CTA, float32 weight: a chunk's loads feed only 8·EB
      // FMAs, so the pass is bound by load latency. The weights of kAhead
      // chunks are loaded before any of their FMAs; every logit still adds
      // its chunks in lane order (c = lane, lane + 32, ...) and a chunk's
      // elements in order. (For a quantized weight, whose chunks also need
      // their block parameters and a decode, loading ahead measured slower:
      // 0.047 -> 0.074 ms at 64 tokens, 128 experts, NF4.)
      constexpr int kAhead = 8;
      for (int c0 = lane; c0 < nchunk; c0 += 32 * kAhead) {
        float wv[kAhead][EB][8];
#pragma unroll
        for (int u = 0; u < kAhead; ++u) {
          const int c = c0 + 32 * u;
#pragma unroll
          for (int j = 0; j < EB; ++j) {
            if (c < nchunk && e0 + j < E) {
              gate_chunk8<QT>(a, (uint64_t)(e0 + j) * H + 8ull * c, wv[u][j]);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) wv[u][j][i] = 0.0f;
            }
          }
        }
#pragma unroll
        for (int u = 0; u < kAhead; ++u) {
          const int c = c0 + 32 * u;
          if (c < nchunk) {
            const float4 x0 = *reinterpret_cast<const float4*>(xs + 4 * c);
            const float4 x1 = *reinterpret_cast<const float4*>(xs + 4 * nchunk + 4 * c);
            const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int j = 0; j < EB; ++j)
#pragma unroll
              for (int i = 0; i < 8; ++i) acc[0][j] = __fmaf_rn(xv[i], wv[u][j][i], acc[0][j]);
          }
        }
      }
    } else if constexpr (TT == 1) {
#pragma unroll 2
      for (int c = lane; c < nchunk; c += 32) {
        float wv[EB][8];
#pragma unroll
        for (int j = 0; j < EB; ++j) {
          if (e0 + j < E) {
            gate_chunk8<QT>(a, (uint64_t)(e0 + j) * H + 8ull * c, wv[j]);
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) wv[j][i] = 0.0f;
          }
        }
        const float4 x0 = *reinterpret_cast<const float4*>(xs + 4 * c);
        const float4 x1 = *reinterpret_cast<const float4*>(xs + 4 * nchunk + 4 * c);
        const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int j = 0; j < EB; ++j)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[0][j] = __fmaf_rn(xv[i], wv[j][i], acc[0][j]);
      }
    } else {
#pragma unroll 2
      for (int c = lane; c < nchunk; c += 32) {
        float wv[EB][8];
#pragma unroll
        for (int j = 0; j < EB; ++j) {
          if (e0 + j < E) {
            gate_chunk8<QT>(a, (uint64_t)(e0 + j) * H + 8ull * c, wv[j]);
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) wv[j][i] = 0.0f;
          }
        }
        // One packed FMA (two independent fused multiply-adds, one rounding
        // each) advances the chains of tokens 2u and 2u+1 by element i: every
        // logit still adds its products in element order.
#pragma unroll
        for (int u = 0; u < TT / 2; ++u) {
          float xv[4][4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 v = *reinterpret_cast<const float4*>(xs + ((uint64_t)(4 * u + q) * nchunk + c) * 4);
            xv[q][0] = v.x;
            xv[q][1] = v.y;
            xv[q][2] = v.z;
            xv[q][3] = v.w;
          }
#pragma unroll
          for (int j = 0; j < EB; ++j)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int q = i >> 1, o = (i & 1) * 2;
              fma_f32x2(acc[2 * u][j], acc[2 * u + 1][j], xv[q][o], xv[q][o + 1], wv[j][i], wv[j][i],
                        acc[2 * u][j], acc[2 * u + 1][j]);
            }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
      for (int j = 0; j < EB; ++j) {
        float v = acc[t][j];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(kFull, v, off));
        if (lane == 0 && e0 + j < E) lg[t * E + e0 + j] = v;
      }
  }
  __syncthreads();
  // One warp per token of the tile (a warp takes several when the tile has
  // more tokens than the CTA has warps).
  for (int tw = warp; tw < nt; tw += kRouterThreads / 32) {
    const int t = t0 + tw;
    float* l = lg + tw * E;
    float* q = pr + tw * E;
    float m = __int_as_float(0xff800000);
    for (int e = lane; e < E; e += 32) m = fmaxf(m, l[e]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, off));
    for (int e = lane; e < E; e += 32) q[e] = own_expf(__fsub_rn(l[e], m));
    __syncwarp();
    // Sequential sum in expert order, then every lane divides its share.
    float s = 0.0f;
    if (lane == 0)
      for (int e = 0; e < E; ++e) s = __fadd_rn(s, q[e]);
    s = __shfl_sync(kFull, s, 0);
    for (int e = lane; e < E; e += 32) q[e] = __fdiv_rn(q[e], s);
    __syncwarp();
    // Stable descending selection: the largest probability, ties to the
    // lower expert index (what a scan with strict > from the lowest index
    // keeps). Warp-parallel: lane l holds experts l, l+32, ...; each round
    // takes the lane-local best and reduces (value, index) across the warp.
    // A NaN makes that order partial, so then lane 0 scans as the reference
    // does.
    int* sel = reinterpret_cast<int*>(l);  // l[] is free now; sel[j] in its first k words
    bool nan = false;
    for (int e = lane; e < E; e += 32) nan |= q[e] != q[e];
    if (!__any_sync(kFull, nan)) {
      float v[kMaxExperts / 32];
#pragma unroll
      for (int i = 0; i < kMaxExperts / 32; ++i) v[i] = lane + 32 * i < E ? q[lane + 32 * i] : 0.0f;
      uint32_t taken = 0;
      for (int j = 0; j < k; ++j) {
        float bv = 0.0f;
        int be = -1;
#pragma unroll
        for (int i = 0; i < kMaxExperts / 32; ++i) {
          const int e = lane + 32 * i;
          if (e < E && !((taken >> i) & 1u) && (be < 0 || v[i] > bv)) {
            bv = v[i];
            be = e;
          }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
          const float ov = __shfl_xor_sync(kFull, bv, off);
          const int oe = __shfl_xor_sync(kFull, be, off);
          if (oe >= 0 && (be < 0 || ov > bv || (ov == bv && oe < be))) {
            bv = ov;
            be = oe;
          }
        }
        if ((be & 31) == lane) taken |= 1u << (be >> 5);
        if (lane == 0) sel[j] = be;
      }
    } else if (lane == 0) {
      uint32_t taken[kMaxExperts / 32] = {};
      for (int j = 0; j < k; ++j) {
        int best = -1;
        for (int e = 0; e < E; ++e) {
          if ((taken[e >> 5] >> (e & 31)) & 1u) continue;
          if (best < 0 || q[e] > q[best]) best = e;
        }
        taken[best >> 5] |= 1u << (best & 31);
        sel[j] = best;
      }
    }
    __syncwarp();
    if (lane == 0) {
      float ssum = 0.0f;
      for (int j = 0; j < k; ++j) ssum = __fadd_rn(ssum, q[sel[j]]);
      for (int j = 0; j < k; ++j) {
        a.topk_idx[(uint64_t)t * k + j] = sel[j];
        if (a.topk_w) a.topk_w[(uint64_t)t * k + j] = __fdiv_rn(q[sel[j]], ssum);
      }
    }
  }
  const bool big = (int64_t)a.T * k > kSortOneCta;
  if (big) {
    // This CTA's pairs per expert, added to its token group's counts (zero
    // before the router; a group of kSortGroup tokens spans whole tiles).
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += kRouterThreads) off_s[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < nt * k; p += kRouterThreads)
      atomicAdd(&off_s[__ldcg(a.topk_idx + (uint64_t)t0 * k + p)], 1);
    __syncthreads();
    int* grp = a.cta_base + (uint64_t)(t0 / kSortGroup) * E;
    for (int e = threadIdx.x; e < E; e += kRouterThreads)
      if (off_s[e]) atomicAdd(grp + e, off_s[e]);
  }
  __threadfence();  // this thread's outputs, before the CTA is counted done
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(a.done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (!big) {
    permute_block(a.topk_idx, a.T * k, E, a.counts, a.offsets, a.perm_pair, a.inv_pos, hist, off_s);
  } else {
    // Expert-major, group-minor exclusive scan of the group counts: the
    // pairs of token group c with expert e start at base[c][e]. Thread e
    // walks its column of groups twice (total, then running bases).
    const int nc = (a.T + kSortGroup - 1) / kSortGroup;
    for (int e = threadIdx.x; e < E; e += kRouterThreads) {
      int tot = 0;
#pragma unroll 8
      for (int c = 0; c < nc; ++c) tot += __ldcg(a.cta_base + (uint64_t)c * E + e);
      off_s[e + 1] = tot;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      off_s[0] = 0;
      for (int e = 0; e < E; ++e) off_s[e + 1] += off_s[e];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += kRouterThreads) {
      a.counts[e] = off_s[e + 1] - off_s[e];
      int b = off_s[e];
#pragma unroll 8
      for (int c = 0; c < nc; ++c) {
        int* cell = a.cta_base + (uint64_t)c * E + e;
        const int h = __ldcg(cell);
        *cell = b;
        b += h;
      }
    }
    for (int e = threadIdx.x; e <= E; e += kRouterThreads) a.offsets[e] = off_s[e];
  }
  __syncthreads();
  if (threadIdx.x == 0) *a.done = 0u;
}

// Multi-CTA pair sort, second half: CTA c places the pairs of token group c
// (tokens [c G, (c + 1) G), G = kSortGroup) in pair order at the bases the
// router computed, ranking equal experts with match_any as permute_block
// does, so every expert's pairs stay in ascending pair (= token) order.
__global__ void __launch_bounds__(128) scatter_kernel(const int* __restrict__ topk_idx, int T, int k, int E,
                                                      int G, int* __restrict__ cta_base,
                                                      int* __restrict__ perm_pair, int* __restrict__ inv_pos) {
  pdl_wait();  // the router's bases are final
  pdl_launch_dependents();
  __shared__ int base[kMaxExperts];
  const int c = blockIdx.x;
  for (int e = threadIdx.x; e < E; e += blockDim.x) base[e] = cta_base[(uint64_t)c * E + e];
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  const int p0 = c * G * k, p1 = min(T, (c + 1) * G) * k;
  for (int b0 = p0; b0 < p1; b0 += 32) {
    const int p = b0 + lane;
    const bool valid = p < p1;
    const unsigned act = __ballot_sync(kFull, valid);
    if (valid) {
      const int e = topk_idx[p];
      const unsigned peers = __match_any_sync(act, e);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      const int pos = base[e] + rank;
      perm_pair[pos] = p;
      if (inv_pos) inv_pos[p] = pos;
      __syncwarp(act);
      if (rank == 0) base[e] += __popc(peers);
    }
    __syncwarp();
  }
}

template <int TT, int EB>
static cudaError_t launch_router_tt(const RouterArgs& a, int gate_qtype, size_t smem, cudaStream_t stream) {
  const dim3 grid((a.T + TT - 1) / TT);
  auto kn = router_kernel<RIALLM_COMPRESSION_NONE, TT, EB>;
  auto k4 = router_kernel<RIALLM_COMPRESSION_FOUR_BIT, TT, EB>;
  auto k8 = router_kernel<RIALLM_COMPRESSION_EIGHT_BIT, TT, EB>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k4, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k8, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e;
  if (gate_qtype == RIALLM_COMPRESSION_FOUR_BIT) e = launch_pdl(k4, grid, dim3(kRouterThreads), smem, stream, a);
  else if (gate_qtype == RIALLM_COMPRESSION_EIGHT_BIT) e = launch_pdl(k8, grid, dim3(kRouterThreads), smem, stream, a);
  else e = launch_pdl(kn, grid, dim3(kRouterThreads), smem, stream, a);
  if (e != cudaSuccess) return e;
  if ((int64_t)a.T * a.k > kSortOneCta) {
    e = launch_pdl(scatter_kernel, dim3((a.T + kSortGroup - 1) / kSortGroup), dim3(128), 0, stream,
                   (const int*)a.topk_idx, a.T, a.k, a.E, kSortGroup, a.cta_base, a.perm_pair, a.inv_pos);
    if (e != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

int router_tile_tokens(int T, int H) {
  if (T < 512) return 1;
  return H <= 3072 ? 8 : 4;
}

cudaError_t launch_router(const RouterArgs& a, int gate_qtype, cudaStream_t stream) {
  if (a.T <= 0) return cudaSuccess;
  const int TT = router_tile_tokens(a.T, a.H);
  // logits + probabilities of TT tokens, pair-sort histograms, then the
  // staged x rows (16-byte aligned: the first part is padded to a multiple
  // of 4 words).
  const size_t words = ((size_t)2 * TT * a.E + (size_t)(kRouterThreads / 32) * (a.E + 1) + a.E + 1 + 3) & ~(size_t)3;
  const size_t smem = (size_t)TT * a.H * sizeof(float) + words * sizeof(float);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if ((int64_t)a.T * a.k > kSortOneCta && a.cta_base == nullptr) return cudaErrorInvalidValue;
  // Four experts per warp pass once every warp has at least four and a CTA
  // holds a token tile (with one token per CTA the kernel is latency-bound
  // and the wider pass measured slower: 0.068 against 0.052 ms at 64 tokens,
  // 128 experts, NF4 router).
  const bool eb4 = a.E >= 4 * (kRouterThreads / 32) && TT > 1;
  if (TT == 8) return eb4 ? launch_router_tt<8, 4>(a, gate_qtype, smem, stream)
                          : launch_router_tt<8, 1>(a, gate_qtype, smem, stream);
  if (TT == 4) return eb4 ? launch_router_tt<4, 4>(a, gate_qtype, smem, stream)
                          : launch_router_tt<4, 1>(a, gate_qtype, smem, stream);
  return launch_router_tt<1, 1>(a, gate_qtype, smem, stream);
}

// One warp per pair row, 8 rows per CTA; each lane issues up to eight of
// its row's 16-byte loads before their stores (one 16-byte copy per thread
// and a CTA per row left the copy latency-bound at 0.57 of HBM). With
// pair_perm each 16-byte group of 8 bf16 values is reordered to
// [0,4,1,5,2,6,3,7].
__global__ void __launch_bounds__(256) gather_kernel(const void* __restrict__ x, int x_bf16,
                                                     const int* __restrict__ perm_pair, int k, int P, int H,
                                                     void* __restrict__ x_perm, int pair_perm,
                                                     const int* __restrict__ row_begin,
                                                     const int* __restrict__ row_end) {
  // The router's outputs are final once this returns; the expert GEMM that
  // follows reads only the routing counts until it waits for x_perm, so it
  // may start now.
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= P) return;
  // Expert-parallel calls gather only the rows of this rank's experts.
  if (row_begin && (row < __ldg(row_begin) || row >= __ldg(row_end))) return;
  const int esz = x_bf16 ? 2 : 4;
  const int n16 = H * esz / 16;
  const int t = __ldg(perm_pair + row) / k;
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(x) + (uint64_t)t * H * esz);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(x_perm) + (uint64_t)row * H * esz);
  for (int i0 = lane; i0 < n16; i0 += 32 * 8) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (i0 + 32 * u < n16) v[u] = __ldg(src + i0 + 32 * u);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (i0 + 32 * u >= n16) break;
      if (pair_perm) {
        uint4 o;
        o.x = prmt(v[u].x, v[u].z, 0x5410u);
        o.y = prmt(v[u].x, v[u].z, 0x7632u);
        o.z = prmt(v[u].y, v[u].w, 0x5410u);
        o.w = prmt(v[u].y, v[u].w, 0x7632u);
        dst[i0 + 32 * u] = o;
      } else {
        dst[i0 + 32 * u] = v[u];
      }
    }
  }
}

cudaError_t launch_gather(const void* x, bool x_bf16, const int* perm_pair, int k, int P, int H,
                          void* x_perm, bool pair_perm, cudaStream_t stream, const int* row_begin,
                          const int* row_end) {
  if (P == 0) return cudaSuccess;
  const dim3 grid((P + 7) / 8);
  cudaError_t e = launch_pdl(gather_kernel, grid, dim3(256), 0, stream, x, x_bf16 ? 1 : 0, perm_pair, k, P, H,
                             x_perm, (pair_perm && x_bf16) ? 1 : 0, row_begin, row_end);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// One CTA per (token, column slice); 4 columns per thread per step. The token's pairs are
// visited in expert-ascending order (the reference's index_add order,
// src/model.rs:794-811): acc = acc + y * w, one rounding each, from 0.
__global__ void combine_kernel(const float* __restrict__ y_perm, const int* __restrict__ inv_pos,
                               const int* __restrict__ topk_idx, const float* __restrict__ topk_w,
                               int k, int H, const float* __restrict__ shared_y,
                               const float* __restrict__ shared_gate, void* out, int out_bf16,
                               int add_to_out, int e_begin, int e_end, int round_w) {
  // The token's pairs in expert-ascending order (a token's k experts are
  // distinct, so a pair's rank is the number of its pairs with a smaller
  // expert), with their y_perm rows and scaled weights, staged once per CTA.
  __shared__ int s_pos[16];
  __shared__ float s_w[16];
  __shared__ int s_n;
  pdl_wait();  // y_perm comes from the down GEMM
  pdl_launch_dependents();
  const int t = blockIdx.x;
  if (threadIdx.x < 32) {
    const int j = threadIdx.x;
    const int e = j < k ? topk_idx[(uint64_t)t * k + j] : 0x7fffffff;
    // Expert-parallel partial sums keep only this rank's experts.
    const bool mine = j < k && e >= e_begin && e < e_end;
    const unsigned keep = __ballot_sync(0xffffffffu, mine);
    int rank = 0;
    for (int i = 0; i < k; ++i) {
      const int ei = __shfl_sync(0xffffffffu, e, i);
      rank += ((keep >> i) & 1u) && ei < e;
    }
    if (mine) {
      s_pos[rank] = inv_pos[(uint64_t)t * k + j];
      // src/model.rs:800-802: the weight is cast to the activation dtype
      // (bf16 rounding for bf16 activations) before it scales y.
      const float w0 = topk_w[(uint64_t)t * k + j];
      s_w[rank] = round_w ? __bfloat162float(__float2bfloat16_rn(w0)) : w0;
    }
    if (j == 0) s_n = __popc(keep);
  }
  __syncthreads();
  const int n = s_n;
  float gsig = 0.0f;
  if (shared_y) gsig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-shared_gate[t])));
  for (int h = (blockIdx.y * blockDim.x + threadIdx.x) * 4; h < H; h += gridDim.y * blockDim.x * 4) {
    // Eight rows at a time are loaded before their adds; the adds run in
    // expert order.
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int j0 = 0; j0 < n; j0 += 8) {
      float4 y[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj)
        if (j0 + jj < n) y[jj] = *reinterpret_cast<const float4*>(y_perm + (uint64_t)s_pos[j0 + jj] * H + h);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        if (j0 + jj < n) {
          const float w = s_w[j0 + jj];
          a0 = __fadd_rn(a0, __fmul_rn(y[jj].x, w));
          a1 = __fadd_rn(a1, __fmul_rn(y[jj].y, w));
          a2 = __fadd_rn(a2, __fmul_rn(y[jj].z, w));
          a3 = __fadd_rn(a3, __fmul_rn(y[jj].w, w));
        }
      }
    }
    if (shared_y) {
      const float4 s = *reinterpret_cast<const float4*>(shared_y + (uint64_t)t * H + h);
      a0 = __fadd_rn(a0, __fmul_rn(s.x, gsig));
      a1 = __fadd_rn(a1, __fmul_rn(s.y, gsig));
      a2 = __fadd_rn(a2, __fmul_rn(s.z, gsig));
      a3 = __fadd_rn(a3, __fmul_rn(s.w, gsig));
    }
    const uint64_t o = (uint64_t)t * H + h;
    if (out_bf16) {
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(out);
      if (add_to_out) {
        a0 = __fadd_rn(a0, __bfloat162float(ob[o]));
        a1 = __fadd_rn(a1, __bfloat162float(ob[o + 1]));
        a2 = __fadd_rn(a2, __bfloat162float(ob[o + 2]));
        a3 = __fadd_rn(a3, __bfloat162float(ob[o + 3]));
      }
      uint2 pk;
      pk.x = pack_bf16x2(a0, a1);
      pk.y = pack_bf16x2(a2, a3);
      *reinterpret_cast<uint2*>(ob + o) = pk;
    } else {
      float* of = reinterpret_cast<float*>(out);
      if (add_to_out) {
        a0 = __fadd_rn(a0, of[o]);
        a1 = __fadd_rn(a1, of[o + 1]);
        a2 = __fadd_rn(a2, of[o + 2]);
        a3 = __fadd_rn(a3, of[o + 3]);
      }
      *reinterpret_cast<float4*>(of + o) = make_float4(a0, a1, a2, a3);
    }
  }
}

cudaError_t launch_combine(const float* y_perm, const int* inv_pos, const int* topk_idx,
                           const float* topk_w, int T, int k, int H, const float* shared_y,
                           const float* shared_gate, void* out, bool out_bf16, bool add_to_out,
                           cudaStream_t stream, int e_begin, int e_end, bool round_w) {
  if (T == 0) return cudaSuccess;
  const int threads = H >= 1024 ? 256 : 128;
  const dim3 grid(T, (H + threads * 4 - 1) / (threads * 4));
  return launch_pdl(combine_kernel, grid, dim3(threads), 0, stream, y_perm, inv_pos, topk_idx, topk_w, k, H,
                    shared_y, shared_gate, out, out_bf16 ? 1 : 0, add_to_out ? 1 : 0, e_begin, e_end,
                    round_w ? 1 : 0);
}

// ------------------------------------------------- CUDA-core grouped GEMM

// Element e of a tensor in the reference layout, as float32 (same closed
// form as the dequant kernels: NF4 block (e+1)/bs, 8-bit block e/bs).
__device__ __forceinline__ float weight_elem(const riallm_qtensor& w, uint64_t e) {
  if (w.qtype == RIALLM_COMPRESSION_NONE) return __ldg(reinterpret_cast<const float*>(w.data) + e);
  const uint8_t* d = reinterpret_cast<const uint8_t*>(w.data);
  uint32_t code;
  uint64_t b;
  if (w.qtype == RIALLM_COMPRESSION_FOUR_BIT) {
    const uint8_t byte = __ldg(d + (e >> 1));
    code = (e & 1) ? (byte >> 4) & 15u : byte & 15u;
    b = (e + 1) / (uint64_t)w.block_size;
  } else {
    code = __ldg(d + e);
    b = e / (uint64_t)w.block_size;
  }
  const float scale = b < w.n_scales ? __ldg(w.scales + b) : 1.0f;
  const float zero = b < w.n_zero_points ? __ldg(w.zero_points + b) : 0.0f;
  return __fmul_rn(__fsub_rn((float)code, zero), scale);
}

// Tile: 64 weight rows x 16 pairs, K in steps of 32. Block (x = row tile,
// y = enumerated (expert, pair tile)). 256 threads: thread (r, g) owns row
// r and pairs 4g..4g+3.
constexpr int kGR = 64, kGN = 16, kGK = 32;
__global__ void __launch_bounds__(256) grouped_f32_kernel(GroupedF32Args a) {
  __shared__ float ws[kGR][kGK + 1];
  __shared__ float xs[kGN][kGK + 1];
  // Find this block's (expert, pair tile).
  int e = 0, n0 = 0, cnt = a.P, off = 0;
  int y = blockIdx.y;
  if (a.counts) {
    bool found = false;
    for (e = 0; e < a.E; ++e) {
      const int c = a.counts[e];
      const int nt = (c + kGN - 1) / kGN;
      if (y < nt) {
        found = true;
        break;
      }
      y -= nt;
    }
    if (!found) return;
    cnt = a.counts[e];
    off = a.offsets[e];
  } else {
    if (y * kGN >= a.P) return;
  }
  n0 = y * kGN;
  const int r0 = blockIdx.x * kGR;
  const int tid = threadIdx.x;
  const int r = tid & 63, g = tid >> 6;
  const uint64_t wrow0 = (uint64_t)e * a.rows_per_expert + a.row_offset + r0;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < a.K; k0 += kGK) {
    for (int i = tid; i < kGR * kGK; i += 256) {
      const int rr = i / kGK, kk = i % kGK;
      float v = 0.0f;
      if (r0 + rr < a.rows && k0 + kk < a.K) {
        v = weight_elem(a.w, (wrow0 + rr) * (uint64_t)a.K + k0 + kk);
        if (a.round_w_bf16) v = __bfloat162float(__float2bfloat16_rn(v));
      }
      ws[rr][kk] = v;
    }
    for (int i = tid; i < kGN * kGK; i += 256) {
      const int nn = i / kGK, kk = i % kGK;
      float v = 0.0f;
      if (n0 + nn < cnt && k0 + kk < a.K) {
        const uint64_t idx = (uint64_t)(off + n0 + nn) * a.K + k0 + kk;
        v = a.x_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.x)[idx])
                     : reinterpret_cast<const float*>(a.x)[idx];
      }
      xs[nn][kk] = v;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kGK; ++kk) {
      const float wv = ws[r][kk];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = __fmaf_rn(wv, xs[4 * g + j][kk], acc[j]);
    }
    __syncthreads();
  }
  if (r0 + r < a.rows) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + 4 * g + j;
      if (n < cnt) a.y[(uint64_t)(off + n) * a.ldy + a.y_col0 + r0 + r] = acc[j];
    }
  }
}

cudaError_t launch_grouped_f32(const GroupedF32Args& a, cudaStream_t stream) {
  if (a.P == 0) return cudaSuccess;
  dim3 grid((a.rows + kGR - 1) / kGR, (a.P + kGN - 1) / kGN + (a.counts ? a.E : 0));
  grouped_f32_kernel<<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

__global__ void swiglu_kernel(const float* __restrict__ g, int ldg, const float* __restrict__ u, int ldu,
                              void* __restrict__ h, int ldh, int P, int I, int h_bf16) {
  const uint64_t n = (uint64_t)P * I;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t p = i / I, c = i % I;
    const float gv = g[p * ldg + c];
    const float uv = u[p * ldu + c];
    const float hv = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
    if (h_bf16)
      reinterpret_cast<__nv_bfloat16*>(h)[p * ldh + c] = __float2bfloat16_rn(hv);
    else
      reinterpret_cast<float*>(h)[p * ldh + c] = hv;
  }
}

cudaError_t launch_swiglu(const float* g, int ldg, const float* u, int ldu, void* h, int ldh, int P,
                          int I, bool h_bf16, cudaStream_t stream) {
  if (P == 0) return cudaSuccess;
  const uint64_t n = (uint64_t)P * I;
  const uint64_t nb = (n + 255) / 256;
  const int blocks = (int)(nb < 148ull * 16 ? nb : 148ull * 16);
  swiglu_kernel<<<blocks, 256, 0, stream>>>(g, ldg, u, ldu, h, ldh, P, I, h_bf16 ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace rl
