// expert_tc.cu -- grouped expert GEMM on the sm_100a tensor cores with the
// block-quantized weights decoded in registers.
//
// D[row, pair] = sum_c W[row, c] * B[pair, c] for every expert's pairs,
// where W is an NF4 or 8-bit tensor in riallm's layout (src/quantization.rs)
// and B holds bf16 activations in expert-sorted pair order.
//
// Data path per CTA (persistent, one per SM):
//   raw-producer warp : TMA (128-byte swizzle, no multicast) of the packed
//                       codes of two 128-row operands, 128 bytes per row per
//                       stage, into a 3-deep shared-memory ring;
//   B-producer warp   : TMA of the bf16 token tile (N x 64) per K step;
//   8 dequant warps   : read codes from shared memory, decode each weight to
//                       f32 with one LOP3/PRMT and a packed fma.rn.f32x2,
//                       round to bf16 and write the 128 x 64 A tile straight
//                       into tensor memory with tcgen05.st (the A operand
//                       never touches shared memory);
//   MMA warp          : tcgen05.mma kind::f16, A from TMEM, B from shared
//                       memory, f32 accumulators D0/D1 in TMEM;
//   4 epilogue warps  : tcgen05.ld of D0/D1 and either h = silu(D0)*D1
//                       (gate_up, bf16 out) or plain f32 stores (down).
//
// Scale/zero parameters are fetched by the dequant threads themselves with
// cp.async, two stages ahead. NF4 follows the reference decode exactly in
// its indexing: element 63 of a block uses the next block's scale and zero
// (src/quantization.rs:55-72), which for the last block of a row is the
// first block of the next row and, past the tensor's end, scale 1 / zero 0.
//
// Every wait is bounded (common.cuh); on expiry the CTA raises an abort
// flag, every role stops, in-flight copies and MMAs are drained with bounded
// waits, tensor memory is freed and the kernel returns with the status word
// set to RIALLM_ERR_TIMEOUT.
#include "common.cuh"
#include "internal.h"

namespace rl {
namespace tc {

constexpr int kRawStages = 3;
constexpr int kBStages = 4;
constexpr int kAStages = 4;
constexpr int kParamSlots = 4;
constexpr int kNmax = 128;
constexpr int kRawOpBytes = 128 * 128;          // one operand: 128 rows x 128 B
constexpr int kRawStageBytes = 2 * kRawOpBytes;  // 32 KiB
constexpr int kBStageBytes = kNmax * 128;        // 16 KiB
constexpr int kDequantWarps = 8;
constexpr int kEpiWarps = 4;
constexpr int kWarpRaw = 0, kWarpMma = 1, kWarpB = 2, kWarpDq0 = 3, kWarpEpi0 = 11;
constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;  // 480
constexpr int kParamFloats = 8;                          // per thread per slot
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColD0 = 0, kColD1 = 128, kColA = 256;  // A stage s, operand a: kColA + 64 s + 32 a
constexpr int kMaxE = 256;

constexpr int kSmemRaw = 0;
constexpr int kSmemB = kSmemRaw + kRawStages * kRawStageBytes;
constexpr int kSmemPrm = kSmemB + kBStages * kBStageBytes;
constexpr int kSmemBar = kSmemPrm + kParamSlots * 256 * kParamFloats * 4;
constexpr int kNumBars = 2 * kRawStages + 2 * kBStages + 2 * kAStages + 3;
constexpr int kSmemMisc = kSmemBar + 8 * 32;
constexpr int kSmemTab = kSmemMisc + 16;
constexpr int kSmemBytes = kSmemTab + 4 * (4 * kMaxE + 1) + 1024;  // + alignment slack
static_assert(kNumBars <= 32, "barrier area");

struct Params {
  const float* scales;
  const float* zeros;
  uint64_t n_scales, n_zeros;
  int K, rows_per_expert, a1_offset, m_step, m_tiles;
  const int* counts;
  const int* offsets;
  int E;
  int swiglu;
  uint16_t* h_out;
  float* y_out;
  int ld_out;
  int* status;
};

struct Tile {
  int e, m_idx, pos0, nv, N;
  int row0, row1;
};

__device__ __forceinline__ void decode_tile(int t, const int* tile_start, const int* ntn,
                                            const int* cnt_s, const int* off_s, const Params& p,
                                            Tile& ti) {
  int lo = 0, hi = p.E + 1;  // first index with tile_start > t
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (tile_start[mid] <= t) lo = mid + 1;
    else hi = mid;
  }
  const int e = lo - 1;
  const int local = t - tile_start[e];
  const int nt = ntn[e];
  const int m_idx = local / nt, n_idx = local % nt;
  const int n0 = n_idx * kNmax;
  const int nv = min(kNmax, cnt_s[e] - n0);
  ti.e = e;
  ti.m_idx = m_idx;
  ti.pos0 = off_s[e] + n0;
  ti.nv = nv;
  ti.N = nv <= 16 ? 16 : nv <= 32 ? 32 : nv <= 64 ? 64 : 128;
  ti.row0 = e * p.rows_per_expert + m_idx * p.m_step;
  ti.row1 = ti.row0 + p.a1_offset;
}

// Wait used by warp-collective roles: every lane polls, and the warp goes on
// only if all lanes saw the phase complete, so a tcgen05 .sync.aligned
// instruction is never reached by part of a warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int* status) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, status));
}

__device__ __forceinline__ bool wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  return true;
}

// Parameter slot of one dequant thread: floats [0,4) scales, [4,8) zeros.
template <int QT>
__device__ __forceinline__ void issue_params(float* slot, const Params& p, uint64_t f) {
  if (QT == RIALLM_COMPRESSION_FOUR_BIT) {
    if (f + 4 <= p.n_scales) cp_async_16(slot, p.scales + f);
    else
      for (int i = 0; i < 4; ++i) slot[i] = (f + i < p.n_scales) ? __ldg(p.scales + f + i) : 1.0f;
    if (f + 4 <= p.n_zeros) cp_async_16(slot + 4, p.zeros + f);
    else
      for (int i = 0; i < 4; ++i) slot[4 + i] = (f + i < p.n_zeros) ? __ldg(p.zeros + f + i) : 0.0f;
  } else {
    if (f < p.n_scales) cp_async_4(slot, p.scales + f);
    else slot[0] = 1.0f;
    if (f < p.n_zeros) cp_async_4(slot + 4, p.zeros + f);
    else slot[4] = 0.0f;
  }
}

// NF4: decode one 64-element block (8 words, element 8i+j = nibble j of
// word i) into 32 bf16x2 registers. Nibbles are placed in the mantissa of
// an f32 whose value is 128 + q (bits 16-19) or 2048 + q (bits 12-15), and
// v = fma(f, s, -(128 + z) s) (resp. 2048) gives (q - z) s; element 63 uses
// (s2, z2), the next block's parameters.
__device__ __forceinline__ void dequant_nf4_block(const uint32_t (&w)[8], float s, float z, float s2,
                                                  float z2, uint32_t (&out)[32]) {
  const float c16 = -__fmul_rn(__fadd_rn(128.0f, z), s);
  const float c12 = -__fmul_rn(__fadd_rn(2048.0f, z), s);
  const float c12n = -__fmul_rn(__fadd_rn(2048.0f, z2), s2);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t x = w[i];
    const uint32_t s1 = prmt(x, 0u, 0x4104u);  // byte0 -> byte1, byte1 -> byte2
    const uint32_t s2b = prmt(x, 0u, 0x4324u); // byte2 -> byte1, byte3 -> byte2
    const uint32_t s3 = prmt(x, 0u, 0x4034u);  // byte3 -> byte1, byte0 -> byte2
    const float f0 = __uint_as_float(and_or(s3, 0x000F0000u, 0x43000000u));
    const float f1 = __uint_as_float(and_or(s1, 0x0000F000u, 0x45000000u));
    const float f2 = __uint_as_float(and_or(s1, 0x000F0000u, 0x43000000u));
    const float f3 = __uint_as_float(and_or(x, 0x0000F000u, 0x45000000u));
    const float f4 = __uint_as_float(and_or(x, 0x000F0000u, 0x43000000u));
    const float f5 = __uint_as_float(and_or(s2b, 0x0000F000u, 0x45000000u));
    const float f6 = __uint_as_float(and_or(s2b, 0x000F0000u, 0x43000000u));
    const float f7 = __uint_as_float(and_or(s3, 0x0000F000u, 0x45000000u));
    float v0, v1, v2, v3, v4, v5, v6, v7;
    fma_f32x2(v0, v1, f0, f1, s, s, c16, c12);
    fma_f32x2(v2, v3, f2, f3, s, s, c16, c12);
    fma_f32x2(v4, v5, f4, f5, s, s, c16, c12);
    if (i == 7) fma_f32x2(v6, v7, f6, f7, s, s2, c16, c12n);
    else fma_f32x2(v6, v7, f6, f7, s, s, c16, c12);
    out[4 * i + 0] = pack_bf16x2(v0, v1);
    out[4 * i + 1] = pack_bf16x2(v2, v3);
    out[4 * i + 2] = pack_bf16x2(v4, v5);
    out[4 * i + 3] = pack_bf16x2(v6, v7);
  }
}

// 8-bit: 64 bytes (16 words) -> 32 bf16x2 registers. PRMT places byte j in
// bits 8-15 of 0x47000000 (value 32768 + q) and v = fma(f, s, -(32768+z) s).
__device__ __forceinline__ void dequant_int8_64(const uint32_t (&w)[16], float s, float z,
                                                uint32_t (&out)[32]) {
  const float c = -__fmul_rn(__fadd_rn(32768.0f, z), s);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float f0 = __uint_as_float(prmt(w[i], 0x47000000u, 0x7604u));
    const float f1 = __uint_as_float(prmt(w[i], 0x47000000u, 0x7614u));
    const float f2 = __uint_as_float(prmt(w[i], 0x47000000u, 0x7624u));
    const float f3 = __uint_as_float(prmt(w[i], 0x47000000u, 0x7634u));
    float v0, v1, v2, v3;
    fma_f32x2(v0, v1, f0, f1, s, s, c, c);
    fma_f32x2(v2, v3, f2, f3, s, s, c, c);
    out[2 * i + 0] = pack_bf16x2(v0, v1);
    out[2 * i + 1] = pack_bf16x2(v2, v3);
  }
}

template <int QT>
__global__ void __launch_bounds__(kThreads, 1)
    expert_gemm_kernel(const __grid_constant__ CUtensorMap tm_raw,
                       const __grid_constant__ CUtensorMap tm_b16,
                       const __grid_constant__ CUtensorMap tm_b32,
                       const __grid_constant__ CUtensorMap tm_b64,
                       const __grid_constant__ CUtensorMap tm_b128, const Params p) {
  constexpr int KR = QT == RIALLM_COMPRESSION_FOUR_BIT ? 256 : 128;  // K per raw stage
  constexpr int SUB = KR / 64;                                       // A sub-stages per raw stage
  constexpr int BS = QT == RIALLM_COMPRESSION_FOUR_BIT ? 64 : 128;   // quant block
  constexpr int PPS = KR / BS;                                       // param blocks per raw stage

  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* raw = smem + kSmemRaw;
  uint8_t* bst = smem + kSmemB;
  float* prm = reinterpret_cast<float*>(smem + kSmemPrm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + kRawStages;
  uint64_t* b_full = raw_empty + kRawStages;
  uint64_t* b_empty = b_full + kBStages;
  uint64_t* a_full = b_empty + kBStages;
  uint64_t* a_empty = a_full + kAStages;
  uint64_t* d_full = a_empty + kAStages;
  uint64_t* d_empty = d_full + 1;
  uint64_t* drain_bar = d_empty + 1;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(smem + kSmemMisc);
  volatile int* abort_s = reinterpret_cast<volatile int*>(smem + kSmemMisc + 4);
  int* tile_start = reinterpret_cast<int*>(smem + kSmemTab);
  int* ntn = tile_start + kMaxE + 1;
  int* cnt_s = ntn + kMaxE;
  int* off_s = cnt_s + kMaxE;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kRawStages; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kDequantWarps);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&a_full[s], kDequantWarps);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(d_full, 1);
    mbar_init(d_empty, kEpiWarps);
    mbar_init(drain_bar, 1);
    fence_mbar_init();
    *abort_s = 0;
  }
  for (int e = tid; e < p.E; e += kThreads) {
    cnt_s[e] = p.counts[e];
    off_s[e] = p.offsets[e];
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < p.E; ++e) {
      const int nt = (cnt_s[e] + kNmax - 1) / kNmax;
      ntn[e] = nt;
      tile_start[e] = acc;
      acc += nt * p.m_tiles;
    }
    tile_start[p.E] = acc;
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_base_s, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kWarpRaw && lane == 0) {
    tma_prefetch_desc(&tm_raw);
    tma_prefetch_desc(&tm_b16);
    tma_prefetch_desc(&tm_b32);
    tma_prefetch_desc(&tm_b64);
    tma_prefetch_desc(&tm_b128);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  const int total = tile_start[p.E];
  const int n_raw = p.K / KR;
  const int n_sub = p.K / 64;

  if (warp == kWarpRaw) {
    // ------------------------------------------------ raw code producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        Tile ti;
        decode_tile(t, tile_start, ntn, cnt_s, off_s, p, ti);
        for (int c = 0; c < n_raw; ++c, ++it) {
          const int s = it % kRawStages;
          if (!mbar_wait(&raw_empty[s], ((it / kRawStages) & 1) ^ 1, abort_s, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&raw_full[s], kRawStageBytes);
          tma_load_2d(raw + s * kRawStageBytes, &tm_raw, &raw_full[s], c * 128, ti.row0);
          tma_load_2d(raw + s * kRawStageBytes + kRawOpBytes, &tm_raw, &raw_full[s], c * 128, ti.row1);
        }
      }
      // Drain: every issued copy lands before the CTA can exit.
      for (uint32_t j = (it > (uint32_t)kRawStages ? it - kRawStages : 0); j < it; ++j)
        wait_drain(&raw_full[j % kRawStages], (j / kRawStages) & 1);
    }
  } else if (warp == kWarpB) {
    // ---------------------------------------------- B (tokens) producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        Tile ti;
        decode_tile(t, tile_start, ntn, cnt_s, off_s, p, ti);
        const CUtensorMap* tm = ti.N == 16 ? &tm_b16 : ti.N == 32 ? &tm_b32 : ti.N == 64 ? &tm_b64 : &tm_b128;
        const uint32_t bytes = (uint32_t)ti.N * 128u;
        for (int sub = 0; sub < n_sub; ++sub, ++it) {
          const int s = it % kBStages;
          if (!mbar_wait(&b_empty[s], ((it / kBStages) & 1) ^ 1, abort_s, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&b_full[s], bytes);
          tma_load_2d(bst + s * kBStageBytes, tm, &b_full[s], sub * 64, ti.pos0);
        }
      }
      for (uint32_t j = (it > (uint32_t)kBStages ? it - kBStages : 0); j < it; ++j)
        wait_drain(&b_full[j % kBStages], (j / kBStages) & 1);
    }
  } else if (warp == kWarpMma) {
    // -------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t ait = 0, bit = 0, tit = 0;
      bool ok = true, issued = false;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++tit) {
        Tile ti;
        decode_tile(t, tile_start, ntn, cnt_s, off_s, p, ti);
        const uint32_t idesc = idesc_bf16_f32(128, (uint32_t)ti.N);
        if (!mbar_wait(d_empty, (tit & 1) ^ 1, abort_s, p.status)) break;
        tc_fence_after();
        for (int sub = 0; sub < n_sub; ++sub, ++ait, ++bit) {
          const int sa = ait % kAStages, sb = bit % kBStages;
          if (!mbar_wait(&a_full[sa], (ait / kAStages) & 1, abort_s, p.status) ||
              !mbar_wait(&b_full[sb], (bit / kBStages) & 1, abort_s, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(bst + sb * kBStageBytes));
          const uint32_t a0 = tmem + kColA + sa * 64, a1 = a0 + 32;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t acc = (sub | kk) ? 1u : 0u;
            tc_mma_ts(tmem + kColD0, a0 + kk * 8, bdesc + (uint64_t)(kk * 2), idesc, acc);
            tc_mma_ts(tmem + kColD1, a1 + kk * 8, bdesc + (uint64_t)(kk * 2), idesc, acc);
          }
          issued = true;
          tc_commit(&a_empty[sa]);
          tc_commit(&b_empty[sb]);
        }
        if (!ok) break;
        tc_commit(d_full);
      }
      if (issued) {
        tc_commit(drain_bar);
        wait_drain(drain_bar, 0);
      }
    }
  } else if (warp < kWarpEpi0) {
    // ------------------------------------------------- dequant warps
    const int dw = warp - kWarpDq0;       // 0..7
    const int a = dw >> 2;                // operand 0 or 1
    const int q = warp & 3;               // TMEM lane quadrant of this warp
    const int r = 32 * q + lane;          // row inside the 128-row operand
    const int pt = dw * 32 + lane;        // parameter slot owner 0..255
    const int swz = r & 7;
    uint32_t rit = 0, ait = 0;
    bool ok = true;
    const uint64_t blocks_per_row = (uint64_t)(p.K / BS);
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      Tile ti;
      decode_tile(t, tile_start, ntn, cnt_s, off_s, p, ti);
      const uint64_t rg = (uint64_t)(a ? ti.row1 : ti.row0) + r;
      const uint64_t f0 = rg * blocks_per_row;
      issue_params<QT>(prm + ((rit + 0) % kParamSlots) * 256 * kParamFloats + pt * kParamFloats, p, f0);
      cp_async_commit();
      issue_params<QT>(prm + ((rit + 1) % kParamSlots) * 256 * kParamFloats + pt * kParamFloats, p,
                       f0 + PPS);
      cp_async_commit();
      for (int c = 0; c < n_raw; ++c, ++rit) {
        if (c + 2 <= n_raw)
          issue_params<QT>(prm + ((rit + 2) % kParamSlots) * 256 * kParamFloats + pt * kParamFloats, p,
                           f0 + (uint64_t)(c + 2) * PPS);
        cp_async_commit();
        cp_async_wait<1>();
        const int s = rit % kRawStages;
        if (!warp_wait(&raw_full[s], (rit / kRawStages) & 1, abort_s, p.status)) {
          ok = false;
          break;
        }
        const float* P0 = prm + (rit % kParamSlots) * 256 * kParamFloats + pt * kParamFloats;
        const float* P1 = prm + ((rit + 1) % kParamSlots) * 256 * kParamFloats + pt * kParamFloats;
        const uint8_t* rowp = raw + s * kRawStageBytes + a * kRawOpBytes + r * 128;
#pragma unroll 1
        for (int u = 0; u < SUB; ++u, ++ait) {
          uint32_t regs[32];
          if (QT == RIALLM_COMPRESSION_FOUR_BIT) {
            const uint4 c0 = *reinterpret_cast<const uint4*>(rowp + (((2 * u) ^ swz) << 4));
            const uint4 c1 = *reinterpret_cast<const uint4*>(rowp + (((2 * u + 1) ^ swz) << 4));
            const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            const float sc = P0[u], ze = P0[4 + u];
            const float sc2 = u < 3 ? P0[u + 1] : P1[0];
            const float ze2 = u < 3 ? P0[4 + u + 1] : P1[4];
            dequant_nf4_block(w, sc, ze, sc2, ze2, regs);
          } else {
            uint32_t w[16];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint4 cj = *reinterpret_cast<const uint4*>(rowp + (((4 * u + j) ^ swz) << 4));
              w[4 * j + 0] = cj.x;
              w[4 * j + 1] = cj.y;
              w[4 * j + 2] = cj.z;
              w[4 * j + 3] = cj.w;
            }
            dequant_int8_64(w, P0[0], P0[4], regs);
          }
          const int sa = ait % kAStages;
          if (!warp_wait(&a_empty[sa], ((ait / kAStages) & 1) ^ 1, abort_s, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          tmem_st_32x32b_x32(tmem + ((uint32_t)(32 * q) << 16) + kColA + sa * 64 + a * 32, regs);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[sa]);
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[s]);
      }
    }
    cp_async_wait<0>();
  } else {
    // ------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int m = 32 * q + lane;
    uint32_t tit = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++tit) {
      Tile ti;
      decode_tile(t, tile_start, ntn, cnt_s, off_s, p, ti);
      if (!warp_wait(d_full, tit & 1, abort_s, p.status)) break;
      tc_fence_after();
      const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
      for (int n0 = 0; n0 < ti.N; n0 += 16) {
        uint32_t g[16], u[16];
        tmem_ld_32x32b_x16(lane_base + kColD0 + n0, g);
        tmem_ld_32x32b_x16(lane_base + kColD1 + n0, u);
        tmem_wait_ld();
        if (p.swiglu) {
          const int col = ti.m_idx * 128 + m;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (n0 + j < ti.nv) {
              const float gv = __uint_as_float(g[j]), uv = __uint_as_float(u[j]);
              const float hv = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
              const __nv_bfloat16 hb = __float2bfloat16_rn(hv);
              p.h_out[(uint64_t)(ti.pos0 + n0 + j) * p.ld_out + col] = *reinterpret_cast<const uint16_t*>(&hb);
            }
          }
        } else {
          const int col = ti.m_idx * 256 + m;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (n0 + j < ti.nv) {
              float* yrow = p.y_out + (uint64_t)(ti.pos0 + n0 + j) * p.ld_out;
              yrow[col] = __uint_as_float(g[j]);
              yrow[col + 128] = __uint_as_float(u[j]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(d_empty);
    }
  }

  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace tc

cudaError_t launch_tc_gemm(const TcGemmArgs& a, int num_sms, cudaStream_t stream) {
  if (a.P == 0) return cudaSuccess;
  const bool nf4 = a.w.qtype == RIALLM_COMPRESSION_FOUR_BIT;
  const uint64_t row_bytes = nf4 ? (uint64_t)a.K / 2 : (uint64_t)a.K;
  const uint64_t total_rows = (uint64_t)a.E * a.rows_per_expert;
  CUtensorMap tm_raw, tm_b[4];
  if (encode_tensor_map_2d(&tm_raw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w.data, row_bytes, total_rows,
                           row_bytes, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  const uint32_t Ns[4] = {16, 32, 64, 128};
  for (int i = 0; i < 4; ++i)
    if (encode_tensor_map_2d(&tm_b[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.b, (uint64_t)a.K,
                             (uint64_t)a.P, (uint64_t)a.K * 2, 64, Ns[i],
                             CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  tc::Params p{a.w.scales, a.w.zero_points, a.w.n_scales, a.w.n_zero_points, a.K,
               a.rows_per_expert, a.a1_offset, a.m_step, a.m_tiles, a.counts, a.offsets, a.E,
               a.swiglu ? 1 : 0, a.h_out, a.y_out, a.ld_out, a.status};
  auto kern = nf4 ? tc::expert_gemm_kernel<RIALLM_COMPRESSION_FOUR_BIT>
                  : tc::expert_gemm_kernel<RIALLM_COMPRESSION_EIGHT_BIT>;
  // Set the shared-memory opt-in once per device and variant, outside any
  // stream capture (the first call is never captured: it sizes the arena).
  static bool attr_done[64][2] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  bool& done = attr_done[dev & 63][nf4 ? 0 : 1];
  if (!done) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmemBytes);
    if (err != cudaSuccess) return err;
    done = true;
  }
  kern<<<num_sms, tc::kThreads, tc::kSmemBytes, stream>>>(tm_raw, tm_b[0], tm_b[1], tm_b[2], tm_b[3], p);
  return cudaGetLastError();
}

}  // namespace rl
