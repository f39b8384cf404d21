// quant.cu -- NF4 / 8-bit block quantization and dequantization kernels.
//
// Bit-identical to riallm's host loops (src/quantization.rs). Every float
// step uses an explicit round-to-nearest intrinsic so the compiler cannot
// fuse or reorder it. Dequantization is HBM-bound: a warp reads contiguous
// codes and writes contiguous 16-byte vectors. Quantization stages blocks
// in shared memory so that its global loads and stores are coalesced while
// each block is still reduced in the reference's sequential order. Grids
// are sized in multiples of the SM count.
#include "common.cuh"
#include "internal.h"

namespace rl {

__constant__ float kNf4Table[16] = {-1.0f,   -0.6962f, -0.5250f, -0.3900f, -0.2750f, -0.1750f,
                                    -0.0850f, -0.0150f, 0.0f,    0.0150f,  0.0850f,  0.1750f,
                                    0.2750f, 0.3900f,  0.5250f,  0.6962f};

// -------------------------------------------------------------- dequant

struct DqParams {
  const uint8_t* data;
  const float* scales;
  const float* zeros;
  uint64_t n_scales, n_zeros, numel;
  uint32_t block_size;
  int mode;  // riallm_dequant_mode
};

__device__ __forceinline__ float dq_value(const DqParams& p, uint32_t code, uint64_t b, bool nf4) {
  float scale = b < p.n_scales ? __ldg(p.scales + b) : 1.0f;
  float zero = b < p.n_zeros ? __ldg(p.zeros + b) : 0.0f;
  if (p.mode == 0) return __fmul_rn(__fsub_rn((float)code, zero), scale);
  if (nf4) return __fmul_rn(kNf4Table[code], scale);
  return __fadd_rn(__fmul_rn((float)code, scale), zero);
}

template <typename OutT>
__device__ __forceinline__ void store_val(OutT* out, uint64_t i, float v);
template <>
__device__ __forceinline__ void store_val<float>(float* out, uint64_t i, float v) {
  out[i] = v;
}
template <>
__device__ __forceinline__ void store_val<__nv_bfloat16>(__nv_bfloat16* out, uint64_t i, float v) {
  out[i] = __float2bfloat16_rn(v);
}

// NF4 (src/quantization.rs:45-76). Element e takes its code from byte e/2
// (low nibble for even e) and its scale / zero from block (e+1)/block_size:
// the reference advances its scale index after the low nibble of the byte
// that ends a block, so the high nibble there (element 63 of a 64-block)
// already reads the next block, and the tensor's last element falls back
// to scale 1.0 / zero 0.0. Each thread decodes 16 bytes = 32 elements.
template <typename OutT>
__global__ void dequant_nf4_kernel(DqParams p, OutT* __restrict__ out) {
  const uint64_t nchunk = (p.numel + 31) / 32;
  for (uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; c < nchunk;
       c += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t e0 = c * 32;
    uint8_t bytes[16];
    if (e0 + 32 <= p.numel && ((reinterpret_cast<uintptr_t>(p.data) & 15) == 0)) {
      uint4 v = __ldg(reinterpret_cast<const uint4*>(p.data) + c);
      memcpy(bytes, &v, 16);
    } else {
      const uint64_t nb = (p.numel + 1) / 2;
      for (int i = 0; i < 16; ++i) bytes[i] = (e0 / 2 + i < nb) ? p.data[e0 / 2 + i] : 0;
    }
    // Block of element e: (e + 1) / block_size, stepped instead of divided.
    uint64_t b = (e0 + 1) / p.block_size;
    uint32_t r = (uint32_t)(e0 + 1 - b * p.block_size);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const uint64_t e = e0 + i;
      if (e >= p.numel) break;
      uint32_t code = (i & 1) ? (bytes[i >> 1] >> 4) & 15u : bytes[i >> 1] & 15u;
      store_val(out, e, dq_value(p, code, b, true));
      if (++r == p.block_size) {
        r = 0;
        ++b;
      }
    }
  }
}

// 8-bit (src/quantization.rs:79-95): element e uses block e/block_size.
template <typename OutT>
__global__ void dequant_int8_kernel(DqParams p, OutT* __restrict__ out) {
  const uint64_t nchunk = (p.numel + 15) / 16;
  for (uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; c < nchunk;
       c += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t e0 = c * 16;
    uint8_t bytes[16];
    if (e0 + 16 <= p.numel && ((reinterpret_cast<uintptr_t>(p.data) & 15) == 0)) {
      uint4 v = __ldg(reinterpret_cast<const uint4*>(p.data) + c);
      memcpy(bytes, &v, 16);
    } else {
      for (int i = 0; i < 16; ++i) bytes[i] = (e0 + i < p.numel) ? p.data[e0 + i] : 0;
    }
    uint64_t b = e0 / p.block_size;
    uint32_t r = (uint32_t)(e0 - b * p.block_size);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint64_t e = e0 + i;
      if (e >= p.numel) break;
      store_val(out, e, dq_value(p, bytes[i], b, false));
      if (++r == p.block_size) {
        r = 0;
        ++b;
      }
    }
  }
}

template <typename OutT>
__global__ void copy_f32_kernel(const float* __restrict__ src, uint64_t n, OutT* __restrict__ out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    store_val(out, i, src[i]);
}

// Eight consecutive outputs: two 16-byte stores of float32 or one of bf16
// (dst 16-byte aligned).
__device__ __forceinline__ void store8(float* out, uint64_t e0, const float (&v)[8]) {
  float4* o = reinterpret_cast<float4*>(out + e0);
  o[0] = make_float4(v[0], v[1], v[2], v[3]);
  o[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* out, uint64_t e0, const float (&v)[8]) {
  uint4 w;
  w.x = pack_bf16x2(v[0], v[1]);
  w.y = pack_bf16x2(v[2], v[3]);
  w.z = pack_bf16x2(v[4], v[5]);
  w.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(out + e0) = w;
}

// NF4, 64-element blocks (the format's block size), coalesced: thread i of
// the grid-stride loop decodes elements 8i .. 8i+7 from one 4-byte word of
// codes, so a warp reads 128 contiguous bytes and writes 1 KiB (float32) or
// 512 bytes (bf16) contiguous with 16-byte stores. Elements 8i .. 8i+6 use
// block (8i+1)/64 = 8i/64; element 8i+7 uses (8i+8)/64, the next block when
// it is element 63 of its block (src/quantization.rs:55-72). Same arithmetic
// as dq_value. Requires numel % 8 == 0 and 4-/16-byte aligned data / out.
template <typename OutT>
__global__ void __launch_bounds__(256) dequant_nf4_b64_kernel(DqParams p, OutT* __restrict__ out) {
  const uint64_t nw = p.numel / 8;
  const uint32_t* codes = reinterpret_cast<const uint32_t*>(p.data);
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < nw; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t w = __ldg(codes + i);
    const uint64_t b0 = i >> 3, b7 = (8 * i + 8) >> 6;
    const float s0 = b0 < p.n_scales ? __ldg(p.scales + b0) : 1.0f;
    const float z0 = b0 < p.n_zeros ? __ldg(p.zeros + b0) : 0.0f;
    const float s7 = b7 < p.n_scales ? __ldg(p.scales + b7) : 1.0f;
    const float z7 = b7 < p.n_zeros ? __ldg(p.zeros + b7) : 0.0f;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t q = (w >> (4 * j)) & 15u;
      const float s = j == 7 ? s7 : s0, z = j == 7 ? z7 : z0;
      if (p.mode == 0) v[j] = __fmul_rn(__fsub_rn((float)q, z), s);
      else v[j] = __fmul_rn(kNf4Table[q], s);
    }
    store8(out, 8 * i, v);
  }
}

// 8-bit, 128-element blocks, coalesced: thread i decodes elements 8i .. 8i+7
// (one 8-byte load, one block e/128 for all eight).
template <typename OutT>
__global__ void __launch_bounds__(256) dequant_int8_b128_kernel(DqParams p, OutT* __restrict__ out) {
  const uint64_t nw = p.numel / 8;
  const uint2* codes = reinterpret_cast<const uint2*>(p.data);
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < nw; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint2 c = __ldg(codes + i);
    const uint64_t b = i >> 4;
    const float s = b < p.n_scales ? __ldg(p.scales + b) : 1.0f;
    const float z = b < p.n_zeros ? __ldg(p.zeros + b) : 0.0f;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float q = (float)(((j < 4 ? c.x : c.y) >> (8 * (j & 3))) & 255u);
      v[j] = p.mode == 0 ? __fmul_rn(__fsub_rn(q, z), s) : __fadd_rn(__fmul_rn(q, s), z);
    }
    store8(out, 8 * i, v);
  }
}

// (Measured alternatives, both slower on B200 for the 939 M-element Mixtral
// gate_up tensor: four items per thread a grid stride apart, 3.56 against
// 4.45 TB/s for NF4 -> bf16; four consecutive blockDim runs per CTA with
// the four code loads issued first, 3.97 TB/s.)

// --------------------------------------------------------------- quantize

// src/quantization.rs:179-196: nearest code to clamp(v,-1,1), strict < so
// the first minimum wins; a NaN distance never wins (code 0).
__device__ __forceinline__ uint32_t nf4_code(float value) {
  float x = value;
  if (x < -1.0f) x = -1.0f;
  if (x > 1.0f) x = 1.0f;
  float min_dist = 3.402823466e+38f;
  uint32_t q = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float dist = fabsf(__fsub_rn(x, kNf4Table[i]));
    if (dist < min_dist) {
      min_dist = dist;
      q = i;
    }
  }
  return q;
}

// Both quantizers stage a tile of kQBlocks blocks of the input in shared
// memory with coalesced loads (rows padded by one float, so that thread t
// walking block t sequentially hits bank (t + i) % 32), then thread t
// quantizes block t in the reference's element order, and the codes go back
// to global memory coalesced through shared memory.
constexpr int kQBlocks = 128;

__device__ __forceinline__ void stage_tile(const float* __restrict__ v, uint64_t n, uint64_t e_begin,
                                           uint32_t count, uint32_t row, float* tile) {
  // count elements from e_begin into rows of `row` floats (+1 padding).
  const bool vec = ((reinterpret_cast<uintptr_t>(v + e_begin) & 15) == 0) && (count % 4 == 0);
  if (vec) {
    for (uint32_t i = threadIdx.x; i < count / 4; i += blockDim.x) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(v + e_begin) + i);
      const uint32_t e = 4 * i, r = e / row, c = e % row;  // row % 4 == 0: a float4 stays in one row
      float* d = tile + r * (row + 1) + c;
      d[0] = f.x;
      d[1] = f.y;
      d[2] = f.z;
      d[3] = f.w;
    }
  } else {
    for (uint32_t e = threadIdx.x; e < count; e += blockDim.x) tile[(e / row) * (row + 1) + e % row] = v[e_begin + e];
  }
}

// NF4 (src/quantization.rs:132-166): absmax, sequential float32 sum from
// -0.0, mean = sum / len, codes packed two per byte (second element in the
// high nibble; an odd tail pads with code(0.0)).
__global__ void __launch_bounds__(kQBlocks) quant_nf4_kernel(const float* __restrict__ v, uint64_t n,
                                                             uint8_t* __restrict__ data, float* __restrict__ scales,
                                                             float* __restrict__ zeros) {
  __shared__ float tile[kQBlocks * 65];
  __shared__ uint32_t words[kQBlocks * 9];  // 8 code words per block, padded to 9
  const uint64_t nb = (n + 63) / 64;
  const int t = threadIdx.x;
  for (uint64_t b0 = (uint64_t)blockIdx.x * kQBlocks; b0 < nb; b0 += (uint64_t)gridDim.x * kQBlocks) {
    const uint32_t nblk = (uint32_t)min((uint64_t)kQBlocks, nb - b0);
    const uint64_t e_begin = b0 * 64;
    const uint32_t count = (uint32_t)min((uint64_t)nblk * 64, n - e_begin);
    stage_tile(v, n, e_begin, count, 64, tile);
    __syncthreads();
    if ((uint32_t)t < nblk) {
      const uint32_t len = min(64u, count - 64u * t);
      const float* blk = tile + t * 65;
      float abs_max = 0.0f;
      float sum = -0.0f;
      for (uint32_t i = 0; i < len; ++i) {
        const float x = blk[i];
        abs_max = fmaxf(abs_max, fabsf(x));
        sum = __fadd_rn(sum, x);
      }
      scales[b0 + t] = __fdiv_rn(abs_max, 1.0f);
      zeros[b0 + t] = __fdiv_rn(sum, (float)len);
      for (uint32_t wi = 0; wi < 8; ++wi) {
        uint32_t word = 0;
        for (uint32_t k = 0; k < 8; ++k) {
          const uint32_t i = 8 * wi + k;
          // the odd tail's pad nibble is code(0.0); bytes past the data end are not stored
          const uint32_t q = i < len ? nf4_code(blk[i]) : (i == len && (len & 1) ? nf4_code(0.0f) : 0u);
          word |= q << (4 * k);
        }
        words[t * 9 + wi] = word;
      }
    }
    __syncthreads();
    const uint32_t nbytes = (count + 1) / 2;
    uint8_t* dst = data + e_begin / 2;
    for (uint32_t i = t; i < nbytes; i += blockDim.x) {
      const uint32_t blk = i / 32, off = i % 32;
      dst[i] = (uint8_t)(words[blk * 9 + off / 4] >> (8 * (off % 4)));
    }
    __syncthreads();
  }
}

// 8-bit (src/quantization.rs:214-235): scale = (max - min) / 255, zero = min,
// code = clamp(round((v - zero) / scale), 0, 255) with Rust's saturating
// `as u8` (NaN -> 0).
__global__ void __launch_bounds__(kQBlocks / 2) quant_int8_kernel(const float* __restrict__ v, uint64_t n,
                                                                  uint8_t* __restrict__ data,
                                                                  float* __restrict__ scales,
                                                                  float* __restrict__ zeros) {
  constexpr int kB = kQBlocks / 2;  // 64 blocks of 128 per tile
  __shared__ float tile[kB * 129];
  __shared__ uint32_t words[kB * 33];  // 32 code words per block, padded to 33
  const uint64_t nb = (n + 127) / 128;
  const int t = threadIdx.x;
  for (uint64_t b0 = (uint64_t)blockIdx.x * kB; b0 < nb; b0 += (uint64_t)gridDim.x * kB) {
    const uint32_t nblk = (uint32_t)min((uint64_t)kB, nb - b0);
    const uint64_t e_begin = b0 * 128;
    const uint32_t count = (uint32_t)min((uint64_t)nblk * 128, n - e_begin);
    stage_tile(v, n, e_begin, count, 128, tile);
    __syncthreads();
    if ((uint32_t)t < nblk) {
      const uint32_t len = min(128u, count - 128u * t);
      const float* blk = tile + t * 129;
      float mn = __int_as_float(0x7f800000), mx = __int_as_float(0xff800000);
      for (uint32_t i = 0; i < len; ++i) mn = fminf(mn, blk[i]);
      for (uint32_t i = 0; i < len; ++i) mx = fmaxf(mx, blk[i]);
      const float scale = __fdiv_rn(__fsub_rn(mx, mn), 255.0f);
      scales[b0 + t] = scale;
      zeros[b0 + t] = mn;
      for (uint32_t wi = 0; wi < 32; ++wi) {
        uint32_t word = 0;
        for (uint32_t k = 0; k < 4; ++k) {
          const uint32_t i = 4 * wi + k;
          uint32_t q = 0;
          if (i < len) {
            const float r = roundf(__fdiv_rn(__fsub_rn(blk[i], mn), scale));
            q = (r != r || r <= 0.0f) ? 0u : r >= 255.0f ? 255u : (uint32_t)r;
          }
          word |= q << (8 * k);
        }
        words[t * 33 + wi] = word;
      }
    }
    __syncthreads();
    uint8_t* dst = data + e_begin;
    for (uint32_t i = t; i < count; i += blockDim.x) {
      const uint32_t blk = i / 128, off = i % 128;
      dst[i] = (uint8_t)(words[blk * 33 + off / 4] >> (8 * (off % 4)));
    }
    __syncthreads();
  }
}

static int grid_for(uint64_t items, int threads, int num_sms) {
  uint64_t g = (items + threads - 1) / threads;
  uint64_t cap = (uint64_t)num_sms * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

cudaError_t launch_dequant(const riallm_qtensor& t, int mode, void* dst, int dst_dtype,
                           int num_sms, cudaStream_t stream) {
  const int threads = 256;
  if (t.qtype == RIALLM_COMPRESSION_NONE) {
    int g = grid_for(t.numel, threads, num_sms);
    if (dst_dtype == RIALLM_DTYPE_F32)
      copy_f32_kernel<<<g, threads, 0, stream>>>((const float*)t.data, t.numel, (float*)dst);
    else
      copy_f32_kernel<<<g, threads, 0, stream>>>((const float*)t.data, t.numel,
                                                 (__nv_bfloat16*)dst);
    return cudaGetLastError();
  }
  DqParams p{(const uint8_t*)t.data, t.scales, t.zero_points, t.n_scales, t.n_zero_points,
             t.numel, (uint32_t)t.block_size, mode};
  const uintptr_t da = reinterpret_cast<uintptr_t>(t.data), oa = reinterpret_cast<uintptr_t>(dst);
  const bool nf4 = t.qtype == RIALLM_COMPRESSION_FOUR_BIT;
  // The format's own block sizes, whole 8-element groups and aligned
  // buffers take the coalesced kernels; anything else the general ones.
  if (t.numel % 8 == 0 && (oa & 15) == 0 && (da & (nf4 ? 3 : 7)) == 0 && t.block_size == (nf4 ? 64 : 128)) {
    const int g = grid_for(t.numel / 8, threads, num_sms);
    if (nf4) {
      if (dst_dtype == RIALLM_DTYPE_F32)
        dequant_nf4_b64_kernel<<<g, threads, 0, stream>>>(p, (float*)dst);
      else
        dequant_nf4_b64_kernel<<<g, threads, 0, stream>>>(p, (__nv_bfloat16*)dst);
    } else {
      if (dst_dtype == RIALLM_DTYPE_F32)
        dequant_int8_b128_kernel<<<g, threads, 0, stream>>>(p, (float*)dst);
      else
        dequant_int8_b128_kernel<<<g, threads, 0, stream>>>(p, (__nv_bfloat16*)dst);
    }
    return cudaGetLastError();
  }
  if (t.qtype == RIALLM_COMPRESSION_FOUR_BIT) {
    int g = grid_for((t.numel + 31) / 32, threads, num_sms);
    if (dst_dtype == RIALLM_DTYPE_F32)
      dequant_nf4_kernel<<<g, threads, 0, stream>>>(p, (float*)dst);
    else
      dequant_nf4_kernel<<<g, threads, 0, stream>>>(p, (__nv_bfloat16*)dst);
  } else {
    int g = grid_for((t.numel + 15) / 16, threads, num_sms);
    if (dst_dtype == RIALLM_DTYPE_F32)
      dequant_int8_kernel<<<g, threads, 0, stream>>>(p, (float*)dst);
    else
      dequant_int8_kernel<<<g, threads, 0, stream>>>(p, (__nv_bfloat16*)dst);
  }
  return cudaGetLastError();
}

cudaError_t launch_quantize(int qtype, const float* src, uint64_t n, uint8_t* data, float* scales,
                            float* zeros, int num_sms, cudaStream_t stream) {
  if (qtype == RIALLM_COMPRESSION_FOUR_BIT) {
    const uint64_t tiles = ((n + 63) / 64 + kQBlocks - 1) / kQBlocks;
    quant_nf4_kernel<<<grid_for(tiles, 1, num_sms), kQBlocks, 0, stream>>>(src, n, data, scales, zeros);
  } else {
    const uint64_t tiles = ((n + 127) / 128 + kQBlocks / 2 - 1) / (kQBlocks / 2);
    quant_int8_kernel<<<grid_for(tiles, 1, num_sms), kQBlocks / 2, 0, stream>>>(src, n, data, scales, zeros);
  }
  return cudaGetLastError();
}

}  // namespace rl
