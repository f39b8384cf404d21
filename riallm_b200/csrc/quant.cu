// quant.cu -- NF4 / 8-bit block quantization and dequantization kernels.
//
// Bit-identical to riallm's host loops (src/quantization.rs). Every float
// step uses an explicit round-to-nearest intrinsic so the compiler cannot
// fuse or reorder it. HBM-bound: 16-byte loads and stores, grid sized in
// multiples of the SM count.
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

// One thread per 64-element block (src/quantization.rs:132-166): absmax,
// sequential f32 sum from -0.0, mean = sum / len, codes packed two per byte
// (second element in the high nibble; an odd tail pads with code(0.0)).
__global__ void quant_nf4_kernel(const float* __restrict__ v, uint64_t n, uint8_t* __restrict__ data,
                                 float* __restrict__ scales, float* __restrict__ zeros) {
  const uint64_t nb = (n + 63) / 64;
  for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nb;
       b += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t start = b * 64;
    const uint32_t len = (uint32_t)min((uint64_t)64, n - start);
    const float* blk = v + start;
    float abs_max = 0.0f;
    float sum = -0.0f;
    for (uint32_t i = 0; i < len; ++i) {
      float x = blk[i];
      abs_max = fmaxf(abs_max, fabsf(x));
      sum = __fadd_rn(sum, x);
    }
    scales[b] = __fdiv_rn(abs_max, 1.0f);
    zeros[b] = __fdiv_rn(sum, (float)len);
    uint8_t* o = data + start / 2;
    for (uint32_t i = 0; i < len; i += 2) {
      uint32_t q1 = nf4_code(blk[i]);
      uint32_t q2 = nf4_code(i + 1 < len ? blk[i + 1] : 0.0f);
      o[i / 2] = (uint8_t)((q2 << 4) | q1);
    }
  }
}

// One thread per 128-element block (src/quantization.rs:214-235):
// scale = (max - min) / 255, zero = min, code = clamp(round((v - zero) /
// scale), 0, 255) with Rust's saturating `as u8` (NaN -> 0).
__global__ void quant_int8_kernel(const float* __restrict__ v, uint64_t n, uint8_t* __restrict__ data,
                                  float* __restrict__ scales, float* __restrict__ zeros) {
  const uint64_t nb = (n + 127) / 128;
  for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nb;
       b += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t start = b * 128;
    const uint32_t len = (uint32_t)min((uint64_t)128, n - start);
    const float* blk = v + start;
    float mn = __int_as_float(0x7f800000), mx = __int_as_float(0xff800000);
    for (uint32_t i = 0; i < len; ++i) mn = fminf(mn, blk[i]);
    for (uint32_t i = 0; i < len; ++i) mx = fmaxf(mx, blk[i]);
    const float scale = __fdiv_rn(__fsub_rn(mx, mn), 255.0f);
    scales[b] = scale;
    zeros[b] = mn;
    for (uint32_t i = 0; i < len; ++i) {
      float t = roundf(__fdiv_rn(__fsub_rn(blk[i], mn), scale));
      uint8_t q;
      if (t != t || t <= 0.0f) q = 0;
      else if (t >= 255.0f) q = 255;
      else q = (uint8_t)t;
      data[start + i] = q;
    }
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
  const int threads = 128;
  if (qtype == RIALLM_COMPRESSION_FOUR_BIT) {
    quant_nf4_kernel<<<grid_for((n + 63) / 64, threads, num_sms), threads, 0, stream>>>(
        src, n, data, scales, zeros);
  } else {
    quant_int8_kernel<<<grid_for((n + 127) / 128, threads, num_sms), threads, 0, stream>>>(
        src, n, data, scales, zeros);
  }
  return cudaGetLastError();
}

}  // namespace rl
