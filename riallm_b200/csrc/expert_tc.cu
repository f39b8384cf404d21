// expert_tc.cu -- grouped expert GEMM on the sm_100a tensor cores with the
// block-quantized weights decoded in registers.
//
// D[row, pair] = sum_c W[row, c] * B[pair, c] for every expert's pairs,
// where W is an NF4 or 8-bit tensor in riallm's layout (src/quantization.rs)
// and B holds bf16 activations in expert-sorted pair order.
//
// Data path per CTA (persistent, one per SM):
//   producer warp     : TMA (128-byte swizzle, no multicast) of the packed
//                       codes of two 128-row operands, 128 bytes per row per
//                       stage, into a shared-memory ring (4 stages deep when
//                       every tile holds <= 64 pairs, else 3);
//   token warp        : TMA of the bf16 token tiles (N x 128 K) of every A
//                       stage into its own ring slot, so code prefetch
//                       never waits on MMA progress;
//   8 dequant warps   : read codes from shared memory, decode each weight
//                       (NF4: LOP3 + exact bf16x2 subtract + two bf16x2
//                       FMAs over a split scale; 8-bit: PRMT + fma.rn.f32x2
//                       + bf16 round) and write the 128 x 128 A tiles
//                       straight into tensor memory with tcgen05.st (the A
//                       operand never touches shared memory);
//   4 MMA warps       : tcgen05.mma kind::f16, A from TMEM, B from shared
//                       memory, f32 accumulators in TMEM;
//   4 epilogue warps  : tcgen05.ld of D0/D1 and either h = silu(D0)*D1
//                       (gate_up, bf16 out) or plain f32 stores (down).
// Measured on B200: packed bf16x2 FMA/SUB and LOP3 issue at half rate (one
// warp instruction per 2 cycles per SM sub-partition), so the NF4 decode
// (3 FMA-pipe instructions per 2 weights) is bound near 768 cycles per
// 32768-weight stage; work is spread so that no other role competes.
//
// Scheduling: whole tiles round-robin over the CTAs while two or more full
// waves remain, then stream-K shares of the rest (see Sched), so all SMs
// stream the same number of weight bytes. At decode sizes the gate_up
// launch's producer, after its last load, prefetches into L2 the first
// stages of the down launch that follows (prefetch_next_launch).
//
// NF4 scales and zero points ride in the same TMA stage as the codes (a
// 128-row x 4-block box of each); 8-bit ones are fetched by the dequant
// threads with cp.async, a few stages ahead. NF4 follows the reference
// decode exactly in its indexing: element 63 of a block uses the next
// block's scale and zero (src/quantization.rs:55-72) -- for the stage's
// last block that is the next stage's first (a global load at stage
// start), for a row's last block the next row's first block, or past the
// tensor's end scale 1 / zero 0.
//
// MMA issue: several issuer warps each own one accumulator, because MMAs
// issued from different warps overlap: four when tiles are at most 64
// pairs wide (operand x K half: every sub-stage each issues the 2 K-steps
// of its half) and two (one per operand) when tiles are 128 wide; the
// epilogue adds the K halves. A tcgen05.commit or a barrier wait plus
// fence costs an issuer about as much as an MMA, so the A ring is organised
// in stages of 128 K (two 64-K sub-stages per operand) and the token
// producer arrives on the same "full" barrier as the dequant warps (with
// its TMA byte count): per stage an issuer does one wait, one fence, its
// MMAs (fully unrolled) and one commit.
//
// Tensor memory (512 columns): the accumulators from column 0 (4 x 32
// when every tile of the launch holds at most 32 pairs, 4 x 64 for other
// tiles of at most 64, 2 x 128 for wider ones), then a ring of A stages of
// 128 columns each (operand 0 then operand 1; 64 columns = 128 bf16): three
// stages behind 4 x 32 accumulators, two otherwise.
//
// Every wait is bounded (common.cuh); on expiry the CTA raises an abort
// flag, every role stops, in-flight copies and MMAs are drained with bounded
// waits, tensor memory is freed and the kernel returns with the status word
// set to RIALLM_ERR_TIMEOUT.
#include "common.cuh"
#include "internal.h"

namespace rl {
namespace tc {

constexpr int kRawStages = 4;                    // raw ring: 4 stages for narrow launches, 3 for wide
constexpr int kBRegionBytes = 64 * 1024;         // token ring: 2 stages x 2 boxes x N x 128 B
constexpr int kAStages = 3;                      // A ring: up to 3 stages of 128 K (4 x 64 K sub-stages)
constexpr int kParamSlots = 6;                   // 8-bit parameter ring (cp.async)
constexpr int kParamAhead = 4;                   // stages prefetched ahead
constexpr int kNmax = 128;
constexpr int kRawOpBytes = 128 * 128;           // one operand: 128 rows x 128 B of codes
constexpr int kRawPrmBytes = 128 * 16;           // one operand's 4 scales (or zeros) per row
constexpr int kRawStageBytes = 2 * kRawOpBytes + 4 * kRawPrmBytes;  // 40 KiB
constexpr int kMmaWarps = 4;
constexpr int kMergeBuf = 64 * 1024;             // split-tile merge staging buffer (2, in the rings)
constexpr int kDequantWarps = 8;
constexpr int kEpiWarps = 4;
constexpr int kWarpProd = 0, kWarpBProd = 1, kWarpMma0 = 2, kWarpDq0 = kWarpMma0 + kMmaWarps,
              kWarpEpi0 = kWarpDq0 + kDequantWarps;
constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;  // 576
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxE = 256;

constexpr int kSmemRaw = 0;
// The token ring follows the raw ring: at 4 x 40 KiB for narrow launches
// (3 token stages of <= 16 KiB), at 3 x 40 KiB for wide ones (2 of 32 KiB).
constexpr int kNarrowBBytes = 3 * 2 * 64 * 128;
constexpr int kSmemPrm = (kRawStages * kRawStageBytes + kNarrowBBytes) > ((kRawStages - 1) * kRawStageBytes + kBRegionBytes)
                             ? kRawStages * kRawStageBytes + kNarrowBBytes
                             : (kRawStages - 1) * kRawStageBytes + kBRegionBytes;
constexpr int kSmemBar = kSmemPrm + kParamSlots * 256 * 2 * 4;
constexpr int kNumBars = 2 * kRawStages + 2 * kAStages + 2 + kMmaWarps + 4;
constexpr int kSmemMisc = kSmemBar + 8 * 40;
constexpr int kSmemTab = kSmemMisc + 16;
constexpr int kSmemBytes = kSmemTab + 4 * (4 * kMaxE + 1) + 1024;  // + alignment slack
static_assert(kNumBars <= 40, "barrier area");
static_assert(kSmemBytes <= 227 * 1024, "shared memory");

struct Params {
  const float* scales;
  const float* zeros;
  uint64_t n_scales, n_zeros;
  int K, rows_per_expert, a1_offset, m_step, m_tiles;
  const int* counts;
  const int* offsets;
  int E;
  int swiglu;
  int h_pair_perm;
  uint16_t* h_out;
  float* y_out;
  int ld_out;
  int* status;
  int d_cols;     // 64 or 128 accumulator columns per operand
  float* sk_ws;   // split-tile partial sums, one [2][d_cols][128] f32 slot per CTA; null: whole tiles
  int* sk_flags;  // one counter per CTA, zero between launches
  // Bound (ns) of a split-tile owner's wait for the other CTAs' partial
  // sums, and a count added to the awaited value (0; the test hook
  // riallm_cuda_ctx_expire_next_wait sets one that is never reached, so the
  // bounded wait expires and the launch reports RIALLM_ERR_TIMEOUT).
  uint64_t flag_wait_ns;
  int flag_extra;
  // The next launch's shape, for the L2 prefetch of its first stages
  // (pf_K == 0: no prefetch).
  int pf_K, pf_rows_per_expert, pf_a1_offset, pf_m_step, pf_m_tiles, pf_sk;
};

struct Tile {
  int e, m_idx, pos0, nv, N;
  int row0, row1;
};

// Position in a ring of n stages: stage index and the parity of its
// current use.
struct RingPos {
  int s = 0;
  uint32_t ph = 0;
  __device__ __forceinline__ void next(int n) {
    if (++s == n) {
      s = 0;
      ph ^= 1u;
    }
  }
};

// The raw stages [r0, r1) of tile t.
struct Item {
  Tile ti;
  int t, r0, r1;
};

// Work of one CTA. Without a partial-sum workspace: whole tiles b, b + G,
// b + 2G, ... With one (stream-K): the same whole-tile rounds while at
// least two full waves of tiles remain, then the remaining tiles' W =
// tiles x raw-stages units are cut into G equal contiguous shares
// [W b / G, W (b+1) / G), so every CTA streams the same number of weight
// bytes whatever the tile count. A tile cut by a share boundary is finished
// by the CTA holding its first raw stage (its last item), which adds the
// partial sums the other CTAs published (their first split item). A CTA
// only ever waits at its last item, after publishing its own partial, so
// the waits cannot form a cycle.
struct Sched {
  uint64_t w, w1;    // stream-K units left: [w, w1)
  int t, t_end;      // whole tiles left: t, t + G, ... < t_end
  int sk_tile0;      // first tile of the stream-K region
  int n_raw;
  __device__ __forceinline__ void init(bool sk, int total, int n_raw_) {
    n_raw = n_raw_;
    t = blockIdx.x;
    const int G = gridDim.x;
    const int rounds = total / G >= 2 ? total / G - 1 : 0;
    sk_tile0 = sk ? rounds * G : total;
    t_end = sk_tile0;
    const uint64_t W = (uint64_t)(total - sk_tile0) * n_raw;
    w = W * blockIdx.x / G;
    w1 = W * (blockIdx.x + 1) / G;
  }
};

// The CTAs after an owner whose stream-K shares start inside the owner's
// tile (tile_end, in stream-K units), in CTA (= K) order; CTAs with empty
// shares are skipped. next() returns gridDim.x when there are no more.
struct ContribIter {
  uint64_t b2;
  __device__ __forceinline__ uint64_t next(uint64_t W, uint64_t G, uint64_t tile_end) {
    while (b2 < G) {
      const uint64_t c = b2++;
      const uint64_t s0 = W * c / G;
      if (s0 >= tile_end) {
        b2 = G;
        return G;
      }
      if (W * (c + 1) / G != s0) return c;
    }
    return G;
  }
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

__device__ __forceinline__ bool sched_next(Sched& sc, Item& it, const int* tile_start, const int* ntn,
                                           const int* cnt_s, const int* off_s, const Params& p) {
  if (sc.t < sc.t_end) {
    it.t = sc.t;
    it.r0 = 0;
    it.r1 = sc.n_raw;
    sc.t += gridDim.x;
  } else {
    if (sc.w >= sc.w1) return false;
    const int lt = (int)(sc.w / (uint64_t)sc.n_raw);
    it.t = sc.sk_tile0 + lt;
    it.r0 = (int)(sc.w - (uint64_t)lt * sc.n_raw);
    const uint64_t left = sc.w1 - sc.w;
    it.r1 = left < (uint64_t)(sc.n_raw - it.r0) ? it.r0 + (int)left : sc.n_raw;
    sc.w += (uint64_t)(it.r1 - it.r0);
  }
  decode_tile(it.t, tile_start, ntn, cnt_s, off_s, p, it.ti);
  return true;
}

// Bounded wait until *flag >= target (another CTA's partial sums are
// published); false on abort or after limit_ns.
__device__ __forceinline__ bool wait_flag(const int* flag, int target, volatile int* abort, int* status,
                                          uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v >= target) return true;
    if ((it & 15u) == 15u) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        *abort = 1;
        atomicExch(status, 6 /* RIALLM_ERR_TIMEOUT */);
        return false;
      }
    }
    __nanosleep(64);
  }
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
  while (!mbar_try_wait_suspend(bar, parity, 2000u))
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  return true;
}

// 8-bit parameter slot of one dequant thread: (scale, zero) of one block.
__device__ __forceinline__ void issue_params_int8(float* slot, const Params& p, uint64_t f) {
  if (f < p.n_scales) cp_async_4(slot, p.scales + f);
  else slot[0] = 1.0f;
  if (f < p.n_zeros) cp_async_4(slot + 1, p.zeros + f);
  else slot[1] = 0.0f;
}

__device__ __forceinline__ uint32_t fma_bf16x2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t sub_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint16_t bf16_bits(float f) {
  const __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<const uint16_t*>(&b);
}

// Block parameters as bf16 pairs: s = hi + lo (hi = bf16(s), lo =
// bf16(s - hi), together ~16 significant bits) and c = bf16(-z s). Two
// blocks are split at once: the result's low halves belong to (s0, z0), the
// high halves to (s1, z1).
struct Bf16Pair {
  uint32_t hi, lo, c;
};
__device__ __forceinline__ Bf16Pair split_params2(float s0, float z0, float s1, float z1) {
  Bf16Pair r;
  r.hi = pack_bf16x2(s0, s1);
  const float h0 = __uint_as_float(r.hi << 16), h1 = __uint_as_float(r.hi & 0xffff0000u);
  r.lo = pack_bf16x2(__fsub_rn(s0, h0), __fsub_rn(s1, h1));
  r.c = pack_bf16x2(__fmul_rn(-z0, s0), __fmul_rn(-z1, s1));
  return r;
}
__device__ __forceinline__ uint32_t lo_lo(uint32_t a, uint32_t b) { return prmt(a, b, 0x5410u); }
__device__ __forceinline__ uint32_t hi_hi(uint32_t a, uint32_t b) { return prmt(a, b, 0x7632u); }
__device__ __forceinline__ uint32_t lo_hi(uint32_t a, uint32_t b) { return prmt(a, b, 0x7610u); }

// NF4: decode half (4 words, 32 elements) of a 64-element block into 16
// bf16x2 registers (element 8i+j is nibble j of word i). Register 4i+j
// holds elements 8i+j (low half) and 8i+j+4 (high half): one LOP3 of
// (word >> 4j) against 0x43004300 gives bf16 values 128+q for both, an exact
// subtraction gives q, and v = q*hi + (q*lo + c) gives (q - z) s to ~2^-17
// before the final rounding, i.e. the bf16 rounding of the reference's
// float32 value except at exact ties. Consumers of these A tiles therefore
// see K permuted inside every group of 8 as [0,4,1,5,2,6,3,7] and the B
// operand is stored the same way. (hi2, lo2, c2) carry the block's
// parameters in both halves; (hiL, loL, cL) the block's in the low half and
// the next block's in the high half, used in the second half's last
// register, whose high half is element 63.
template <bool kSecondHalf>
__device__ __forceinline__ void dequant_nf4_half(const uint4 w4, uint32_t hi2, uint32_t lo2, uint32_t c2,
                                                 uint32_t hiL, uint32_t loL, uint32_t cL,
                                                 uint32_t (&out)[16]) {
  const uint32_t m128 = 0x43004300u;
  const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t q = sub_bf16x2(and_or(w[i] >> (4 * j), 0x000F000Fu, m128), m128);
      if (kSecondHalf && i == 3 && j == 3)
        out[4 * i + j] = fma_bf16x2(q, hiL, fma_bf16x2(q, loL, cL));
      else
        out[4 * i + j] = fma_bf16x2(q, hi2, fma_bf16x2(q, lo2, c2));
    }
  }
}

// 8-bit: 32 bytes (8 words, 32 elements) -> 16 bf16x2 registers. PRMT
// places byte j in bits 8-15 of 0x47000000 (value 32768 + q) and
// v = fma(f, s, -(32768+z) s).
__device__ __forceinline__ void dequant_int8_half(const uint4 a4, const uint4 b4, float s, float z,
                                                  uint32_t (&out)[16]) {
  const float c = -__fmul_rn(__fadd_rn(32768.0f, z), s);
  const uint32_t w[8] = {a4.x, a4.y, a4.z, a4.w, b4.x, b4.y, b4.z, b4.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
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

// One A stage of MMAs for one issuer: sub-stages u = 0, 1 (64 K each) and
// K steps kk0 .. kk0 + NKK - 1 of each, accumulating into d (the item's
// first MMA overwrites).
template <int NKK>
__device__ __forceinline__ void issue_stage(uint32_t d, uint32_t a_k, uint64_t b0_k, uint64_t b1_k,
                                            uint32_t idesc, bool first) {
#pragma unroll
  for (int u = 0; u < 2; ++u) {
#pragma unroll
    for (int i = 0; i < NKK; ++i)
      tc_mma_ts(d, a_k + u * 32 + i * 8, (u ? b1_k : b0_k) + (uint64_t)(i * 2), idesc,
                (first && u == 0 && i == 0) ? 0u : 1u);
  }
}

// Raw stages of the next launch prefetched into L2 per CTA.
constexpr int kPfStages = 2;

// The next expert GEMM launch (same weight format) starts on SMs as this
// launch's CTAs exit, and its first weight bytes then come from HBM after
// its prologue. This CTA's producer, once its own loads are all issued,
// works out the first item the same CTA index gets in the next launch (the
// same schedule as Sched over that launch's tiles: ntn is shared, since
// both launches tile the same pairs) and prefetches that item's first
// kPfStages raw stages -- codes and, for NF4, scales and zero points --
// into L2. A prefetch only warms the cache; results do not depend on it.
template <bool kNF4, int KR, int PPS>
__device__ __forceinline__ void prefetch_next_launch(const Params& p, const int* ntn,
                                                     const CUtensorMap* raw, const CUtensorMap* scl,
                                                     const CUtensorMap* zer) {
  const int n_raw = p.pf_K / KR;
  int total = 0;
  for (int e = 0; e < p.E; ++e) total += ntn[e] * p.pf_m_tiles;
  if (total == 0 || n_raw == 0) return;
  const int G = gridDim.x, b = blockIdx.x;
  const int rounds = total / G >= 2 ? total / G - 1 : 0;
  const int sk_tile0 = p.pf_sk ? rounds * G : total;
  int t, r0;
  if (b < sk_tile0) {
    t = b;
    r0 = 0;
  } else {
    const uint64_t W = (uint64_t)(total - sk_tile0) * n_raw;
    const uint64_t w = W * b / G, w1 = W * (b + 1) / G;
    if (w >= w1) return;
    const int lt = (int)(w / (uint64_t)n_raw);
    t = sk_tile0 + lt;
    r0 = (int)(w - (uint64_t)lt * n_raw);
  }
  int e = 0, start = 0;
  for (; e < p.E; ++e) {
    const int n = ntn[e] * p.pf_m_tiles;
    if (t < start + n) break;
    start += n;
  }
  if (e >= p.E) return;
  const int m_idx = (t - start) / ntn[e];
  const int row0 = e * p.pf_rows_per_expert + m_idx * p.pf_m_step;
  const int row1 = row0 + p.pf_a1_offset;
  const int r1 = min(n_raw, r0 + kPfStages);
  for (int c = r0; c < r1; ++c) {
    tma_prefetch_l2_2d(raw, c * 128, row0);
    tma_prefetch_l2_2d(raw, c * 128, row1);
    if (kNF4) {
      tma_prefetch_l2_2d(scl, c * PPS, row0);
      tma_prefetch_l2_2d(zer, c * PPS, row0);
      tma_prefetch_l2_2d(scl, c * PPS, row1);
      tma_prefetch_l2_2d(zer, c * PPS, row1);
    }
  }
}

template <int QT>
__global__ void __launch_bounds__(kThreads, 1)
    expert_gemm_kernel(const __grid_constant__ CUtensorMap tm_raw,
                       const __grid_constant__ CUtensorMap tm_scl,
                       const __grid_constant__ CUtensorMap tm_zer,
                       const __grid_constant__ CUtensorMap tm_b16,
                       const __grid_constant__ CUtensorMap tm_b32,
                       const __grid_constant__ CUtensorMap tm_b64,
                       const __grid_constant__ CUtensorMap tm_b128,
                       const __grid_constant__ CUtensorMap tm_nraw,
                       const __grid_constant__ CUtensorMap tm_nscl,
                       const __grid_constant__ CUtensorMap tm_nzer, const Params p) {
  constexpr bool kNF4 = QT == RIALLM_COMPRESSION_FOUR_BIT;
  constexpr int KR = kNF4 ? 256 : 128;  // K per raw stage (128 code bytes per row)
  constexpr int AS_PER_RAW = KR / 128;  // A stages (128 K each) per raw stage
  constexpr int BS = kNF4 ? 64 : 128;   // quant block
  constexpr int PPS = KR / BS;          // quant blocks per raw stage

  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* raw = smem + kSmemRaw;
  // Narrow launches (every tile <= 64 pairs): 4 issuers, accumulator of
  // issuer j = (operand j&1, K half j>>1) at column acc_cols j. Wide
  // launches: 2 issuers, accumulator of operand j at column 128 j.
  const bool narrow = p.d_cols == 64;
  const int n_rs = narrow ? kRawStages : kRawStages - 1;  // raw ring depth
  uint8_t* bst = smem + n_rs * kRawStageBytes;
  float* prm = reinterpret_cast<float*>(smem + kSmemPrm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + kRawStages;
  uint64_t* full = raw_empty + kRawStages;   // A stage stored + its token tiles landed
  uint64_t* empty = full + kAStages;         // the stage's MMAs completed
  uint64_t* d_full = empty + kAStages;
  uint64_t* d_empty = d_full + 1;
  uint64_t* drain_bar = d_empty + 1;         // one per MMA issuer
  uint64_t* mg_full = drain_bar + kMmaWarps; // split-tile merge: staging buffer b landed
  uint64_t* mg_empty = mg_full + 2;          // staging buffer b read by the four epilogue warps
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(smem + kSmemMisc);
  volatile int* abort_s = reinterpret_cast<volatile int*>(smem + kSmemMisc + 4);
  int* max_nv_s = reinterpret_cast<int*>(smem + kSmemMisc + 8);
  int* tile_start = reinterpret_cast<int*>(smem + kSmemTab);
  int* ntn = tile_start + kMaxE + 1;
  int* cnt_s = ntn + kMaxE;
  int* off_s = cnt_s + kMaxE;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // The next expert GEMM may queue now; its CTAs take SMs as these exit.
  pdl_launch_dependents();
  const int n_iss = narrow ? 4 : 2;
  const uint32_t b_box = narrow ? 64u * 128u : 128u * 128u;  // one 64-K token box
  const uint32_t b_stage = 2 * b_box;

  if (tid == 0) {
    for (int s = 0; s < kRawStages; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kDequantWarps);
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&full[s], kDequantWarps + 1);
      mbar_init(&empty[s], n_iss);
    }
    mbar_init(d_full, n_iss);
    mbar_init(d_empty, kEpiWarps);
    for (int i = 0; i < kMmaWarps; ++i) mbar_init(&drain_bar[i], 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&mg_full[b], 1);
      mbar_init(&mg_empty[b], kEpiWarps);
    }
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
    int mx = 0;
    for (int e = 0; e < p.E; ++e) mx = max(mx, min(cnt_s[e], kNmax));
    *max_nv_s = mx;
  }
  if (warp == kWarpMma0) {
    tmem_alloc(tmem_base_s, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kWarpProd && lane == 0) {
    tma_prefetch_desc(&tm_raw);
    if (kNF4) {
      tma_prefetch_desc(&tm_scl);
      tma_prefetch_desc(&tm_zer);
    }
  }
  if (warp == kWarpBProd && lane == 0) {
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
  const bool sk = p.sk_ws != nullptr;
  // TMEM: accumulators from column 0, then the A ring. Narrow launches whose
  // tiles all hold <= 32 pairs use 32-column accumulators (4 x 32) and
  // three A stages; other narrow launches 4 x 64 and two; wide ones 2 x 128
  // and two.
  const bool small_n = narrow && *max_nv_s <= 32;
  const uint32_t acc_cols = narrow ? (small_n ? 32u : 64u) : 128u;
  const int n_ring = small_n ? 3 : 2;
  const uint32_t col_a = narrow ? 4u * acc_cols : 256u;

  if (warp == kWarpProd) {
    // ------------------------------------------- producer: codes (+ NF4 params)
    if (lane == 0) {
      uint32_t it = 0;
      RingPos rr;
      bool ok = true;
      const uint32_t stage_bytes = kNF4 ? (uint32_t)kRawStageBytes : (uint32_t)(2 * kRawOpBytes);
      Sched sc;
      sc.init(sk, total, n_raw);
      Item im;
      while (ok && sched_next(sc, im, tile_start, ntn, cnt_s, off_s, p)) {
        for (int c = im.r0; c < im.r1; ++c, ++it, rr.next(n_rs)) {
          const int s = rr.s;
          if (!mbar_wait(&raw_empty[s], rr.ph ^ 1, abort_s, p.status)) {
            ok = false;
            break;
          }
          uint8_t* st = raw + s * kRawStageBytes;
          mbar_arrive_expect_tx(&raw_full[s], stage_bytes);
          tma_load_2d(st, &tm_raw, &raw_full[s], c * 128, im.ti.row0);
          tma_load_2d(st + kRawOpBytes, &tm_raw, &raw_full[s], c * 128, im.ti.row1);
          if (kNF4) {
            uint8_t* pp = st + 2 * kRawOpBytes;
            tma_load_2d(pp, &tm_scl, &raw_full[s], c * PPS, im.ti.row0);
            tma_load_2d(pp + kRawPrmBytes, &tm_zer, &raw_full[s], c * PPS, im.ti.row0);
            tma_load_2d(pp + 2 * kRawPrmBytes, &tm_scl, &raw_full[s], c * PPS, im.ti.row1);
            tma_load_2d(pp + 3 * kRawPrmBytes, &tm_zer, &raw_full[s], c * PPS, im.ti.row1);
          }
        }
      }
      if (ok && p.pf_K > 0) prefetch_next_launch<kNF4, KR, PPS>(p, ntn, &tm_nraw, &tm_nscl, &tm_nzer);
      // Drain: every issued copy lands before the CTA can exit.
      for (uint32_t j = (it > (uint32_t)n_rs ? it - n_rs : 0); j < it; ++j)
        wait_drain(&raw_full[j % n_rs], (j / n_rs) & 1);
    }
  } else if (warp == kWarpBProd) {
    // ---------------------------------------------- token tile producer
    if (lane == 0) {
      uint32_t ait = 0;
      RingPos rp;
      bool ok = true;
      Sched sc;
      sc.init(sk, total, n_raw);
      Item im;
      pdl_wait();  // token tiles are the previous kernel's output
      while (ok && sched_next(sc, im, tile_start, ntn, cnt_s, off_s, p)) {
        const Tile& ti = im.ti;
        const CUtensorMap* tm = ti.N == 16 ? &tm_b16 : ti.N == 32 ? &tm_b32 : ti.N == 64 ? &tm_b64 : &tm_b128;
        const uint32_t bbytes = (uint32_t)ti.N * 128u;
        for (int as = im.r0 * AS_PER_RAW; as < im.r1 * AS_PER_RAW; ++as, ++ait, rp.next(n_ring)) {
          const int s = rp.s;
          if (!mbar_wait(&empty[s], rp.ph ^ 1, abort_s, p.status)) {
            ok = false;
            break;
          }
          uint8_t* bs = bst + s * b_stage;
          mbar_arrive_expect_tx(&full[s], 2 * bbytes);
          tma_load_2d(bs, tm, &full[s], as * 128, ti.pos0);
          tma_load_2d(bs + b_box, tm, &full[s], as * 128 + 64, ti.pos0);
        }
      }
      // Drain: the last stages' token copies land before the CTA can exit.
      for (uint32_t j = (ait > (uint32_t)n_ring ? ait - n_ring : 0); j < ait; ++j)
        wait_drain(&full[j % n_ring], (j / n_ring) & 1);
    }
  } else if (warp < kWarpDq0) {
    // ------------------------------------------------------- MMA issuers
    const int j = warp - kWarpMma0;
    if (lane == 0 && j < n_iss) {
      const int op = narrow ? (j & 1) : j;        // operand: 0 gate / rows r, 1 up / rows r+128
      const int kk0 = narrow ? 2 * (j >> 1) : 0;  // first K step of this issuer in a sub-stage
      const uint32_t d_col = acc_cols * j;
      RingPos rp;
      uint32_t tit = 0;
      bool ok = true, issued = false;
      Sched sc;
      sc.init(sk, total, n_raw);
      Item im;
      while (ok && sched_next(sc, im, tile_start, ntn, cnt_s, off_s, p)) {
        const uint32_t idesc = idesc_bf16_f32(128, (uint32_t)im.ti.N);
        if (!mbar_wait(d_empty, (tit & 1) ^ 1, abort_s, p.status)) break;
        const int as0 = im.r0 * AS_PER_RAW;
        for (int as = as0; as < im.r1 * AS_PER_RAW; ++as, rp.next(n_ring)) {
          const int s = rp.s;
          if (!mbar_wait(&full[s], rp.ph, abort_s, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_k = tmem + col_a + s * 128 + op * 64 + kk0 * 8;
          const uint64_t b0_k = sdesc_kmajor_sw128(smem_u32(bst + s * b_stage)) + (uint64_t)(kk0 * 2);
          const uint64_t b1_k = sdesc_kmajor_sw128(smem_u32(bst + s * b_stage + b_box)) + (uint64_t)(kk0 * 2);
          if (narrow)
            issue_stage<2>(tmem + d_col, a_k, b0_k, b1_k, idesc, as == as0);
          else
            issue_stage<4>(tmem + d_col, a_k, b0_k, b1_k, idesc, as == as0);
          issued = true;
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(d_full);
        ++tit;
      }
      if (issued) {
        tc_commit(&drain_bar[j]);
        wait_drain(&drain_bar[j], 0);
      }
    }
  } else if (warp < kWarpEpi0) {
    // ------------------------------------------------- dequant warps
    const int dw = warp - kWarpDq0;       // 0..7
    const int a = dw >> 2;                // operand 0 or 1
    const int q = warp & 3;               // TMEM lane quadrant of this warp
    const int r = 32 * q + lane;          // row inside the 128-row operand
    const int pt = dw * 32 + lane;        // 8-bit parameter slot owner 0..255
    const int swz = r & 7;
    uint32_t rit = 0;
    RingPos rp, rr;
    bool ok = true;
    const uint64_t blocks_per_row = (uint64_t)(p.K / BS);
    Sched sc;
    sc.init(sk, total, n_raw);
    Item im;
    while (ok && sched_next(sc, im, tile_start, ntn, cnt_s, off_s, p)) {
      const Tile& ti = im.ti;
      const uint64_t rg = (uint64_t)(a ? ti.row1 : ti.row0) + r;
      const uint64_t f0 = rg * blocks_per_row;
      if (!kNF4) {
        for (int c = 0; c < kParamAhead; ++c) {
          if (im.r0 + c < im.r1)
            issue_params_int8(prm + ((rit + c) % kParamSlots) * 512 + pt * 2, p, f0 + (uint64_t)(im.r0 + c) * PPS);
          cp_async_commit();
        }
      }
      for (int c = im.r0; c < im.r1; ++c, ++rit, rr.next(n_rs)) {
        // NF4: element 63 of the stage's last block takes the parameters of
        // the block after it -- the next stage's first, the next row's first
        // for the row's last stage, or 1.0 / 0.0 past the tensor's end.
        float next_s = 1.0f, next_z = 0.0f;
        if (kNF4) {
          const uint64_t nb = f0 + (uint64_t)(c + 1) * PPS;
          if (nb < p.n_scales) next_s = __ldg(p.scales + nb);
          if (nb < p.n_zeros) next_z = __ldg(p.zeros + nb);
        } else {
          if (c + kParamAhead < im.r1)
            issue_params_int8(prm + ((rit + kParamAhead) % kParamSlots) * 512 + pt * 2, p,
                              f0 + (uint64_t)(c + kParamAhead) * PPS);
          cp_async_commit();
          cp_async_wait<kParamAhead>();
        }
        const int rs = rr.s;
        if (!warp_wait(&raw_full[rs], rr.ph, abort_s, p.status)) {
          ok = false;
          break;
        }
        const uint8_t* st = raw + rs * kRawStageBytes;
        const uint8_t* rowp = st + a * kRawOpBytes + r * 128;
        // NF4: bf16-split parameters of the raw stage's 4 blocks, two per
        // pair: P01 = (block 0, block 1), P23 = (block 2, block 3).
        Bf16Pair P01{}, P23{};
        if (kNF4) {
          const float* pp = reinterpret_cast<const float*>(st + 2 * kRawOpBytes + a * 2 * kRawPrmBytes);
          const float4 sc4 = *reinterpret_cast<const float4*>(pp + r * 4);
          const float4 ze4 = *reinterpret_cast<const float4*>(pp + kRawPrmBytes / 4 + r * 4);
          P01 = split_params2(sc4.x, ze4.x, sc4.y, ze4.y);
          P23 = split_params2(sc4.z, ze4.z, sc4.w, ze4.w);
        }
        float sc8 = 0.f, ze8 = 0.f;
        if (!kNF4) {
          const float* sl = prm + (rit % kParamSlots) * 512 + pt * 2;
          sc8 = sl[0];
          ze8 = sl[1];
        }
        // NF4: the next sub-stage's codes are loaded one sub-stage ahead.
        uint4 pc0 = make_uint4(0, 0, 0, 0), pc1 = pc0;
        if (kNF4) {
          pc0 = *reinterpret_cast<const uint4*>(rowp + ((0 ^ swz) << 4));
          pc1 = *reinterpret_cast<const uint4*>(rowp + ((1 ^ swz) << 4));
        }
#pragma unroll
        for (int v = 0; v < AS_PER_RAW; ++v, rp.next(n_ring)) {
          const int s = rp.s;
          const uint32_t tdst = tmem + ((uint32_t)(32 * q) << 16) + col_a + s * 128 + a * 64;
          uint32_t regs[16], r32[32];
#pragma unroll
          for (int uu = 0; uu < 2; ++uu) {
            const int u = 2 * v + uu;  // 64-K sub-stage inside the raw stage
            if (kNF4) {
              const uint4 c0 = pc0, c1 = pc1;
              if (u < 3) {
                pc0 = *reinterpret_cast<const uint4*>(rowp + (((2 * u + 2) ^ swz) << 4));
                pc1 = *reinterpret_cast<const uint4*>(rowp + (((2 * u + 3) ^ swz) << 4));
              }
              // Block u's constants in both halves, and (block u, block u+1)
              // for the register holding element 63.
              const Bf16Pair& Pc = (u < 2) ? P01 : P23;
              uint32_t hi2, lo2, c2, hiL, loL, cL;
              if ((u & 1) == 0) {
                hi2 = lo_lo(Pc.hi, Pc.hi); lo2 = lo_lo(Pc.lo, Pc.lo); c2 = lo_lo(Pc.c, Pc.c);
                hiL = Pc.hi; loL = Pc.lo; cL = Pc.c;
              } else {
                hi2 = hi_hi(Pc.hi, Pc.hi); lo2 = hi_hi(Pc.lo, Pc.lo); c2 = hi_hi(Pc.c, Pc.c);
                if (u == 1) {
                  // block 1 (low) with block 2, the low half of P23 (high)
                  hiL = lo_lo(hi2, P23.hi); loL = lo_lo(lo2, P23.lo); cL = lo_lo(c2, P23.c);
                } else {
                  const Bf16Pair Pn = split_params2(next_s, next_z, next_s, next_z);
                  hiL = lo_hi(hi2, Pn.hi); loL = lo_hi(lo2, Pn.lo); cL = lo_hi(c2, Pn.c);
                }
              }
              // Both halves of the sub-stage, then one 32-column store.
              dequant_nf4_half<false>(c0, hi2, lo2, c2, hiL, loL, cL, *reinterpret_cast<uint32_t(*)[16]>(r32));
              dequant_nf4_half<true>(c1, hi2, lo2, c2, hiL, loL, cL, *reinterpret_cast<uint32_t(*)[16]>(r32 + 16));
              if (uu == 0) {
                // The stage's columns are free once its previous MMAs completed.
                if (!warp_wait(&empty[s], rp.ph ^ 1, abort_s, p.status)) {
                  ok = false;
                  break;
                }
                tc_fence_after();
              }
              tmem_st_32x32b_x32(tdst + uu * 32, r32);
            } else {
              const uint4 ca = *reinterpret_cast<const uint4*>(rowp + (((4 * u) ^ swz) << 4));
              const uint4 cb = *reinterpret_cast<const uint4*>(rowp + (((4 * u + 1) ^ swz) << 4));
              dequant_int8_half(ca, cb, sc8, ze8, regs);
              if (uu == 0) {
                if (!warp_wait(&empty[s], rp.ph ^ 1, abort_s, p.status)) {
                  ok = false;
                  break;
                }
                tc_fence_after();
              }
              tmem_st_32x32b_x16(tdst + uu * 32, regs);
              const uint4 cc = *reinterpret_cast<const uint4*>(rowp + (((4 * u + 2) ^ swz) << 4));
              const uint4 cd = *reinterpret_cast<const uint4*>(rowp + (((4 * u + 3) ^ swz) << 4));
              dequant_int8_half(cc, cd, sc8, ze8, regs);
              tmem_st_32x32b_x16(tdst + uu * 32 + 16, regs);
            }
          }
          if (!ok) break;
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);
      }
      if (!kNF4) cp_async_wait<0>();
    }
    cp_async_wait<0>();
  } else {
    // ------------------------------------------------------- epilogue
    // Outputs and the split-tile workspace may still be in use by the
    // previous kernel until it completes.
    pdl_wait();
    const int q = warp & 3;
    const int m = 32 * q + lane;
    const uint64_t G = gridDim.x;
    const uint64_t slot_floats = 2ull * (uint64_t)p.d_cols * 128ull;
    uint32_t tit = 0;
    Sched sc;
    sc.init(sk, total, n_raw);
    const uint64_t W = (uint64_t)(total - sc.sk_tile0) * n_raw;  // stream-K units
    Item im;
    while (sched_next(sc, im, tile_start, ntn, cnt_s, off_s, p)) {
      const Tile& ti = im.ti;
      // part: a later K range of a tile another CTA finishes; owner: this
      // CTA holds the tile's first raw stage but not its last.
      const bool part = sk && im.r0 > 0;
      const bool owner = sk && im.r0 == 0 && im.r1 < n_raw;
      const uint64_t tile_end = (uint64_t)(im.t - sc.sk_tile0 + 1) * n_raw;  // in stream-K units
      if (!warp_wait(d_full, tit & 1, abort_s, p.status)) break;
      tc_fence_after();
      bool ok = true;
      if (owner) {
        // Every CTA whose share starts inside this tile published a partial.
        for (uint64_t b2 = blockIdx.x + 1; b2 < G && ok; ++b2) {
          const uint64_t s0 = W * b2 / G;
          if (s0 >= tile_end) break;
          if (W * (b2 + 1) / G == s0) continue;
          int got = 1;
          if (lane == 0)
            got = wait_flag(p.sk_flags + b2, kEpiWarps + p.flag_extra, abort_s, p.status, p.flag_wait_ns) ? 1 : 0;
          ok = __shfl_sync(0xffffffffu, got, 0) != 0;
        }
        if (!ok) break;
      }
      float* my_slot = part ? p.sk_ws + (uint64_t)blockIdx.x * slot_floats : nullptr;
      const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
      if (owner) {
        // Add the later K ranges' partial sums into this CTA's (K half 0)
        // accumulators in TMEM, in CTA (= K) order: deterministic. This is
        // the CTA's last item, so its raw and token rings are idle: each
        // partial operand ([column][row] f32, N columns) is bulk-copied into
        // one of two staging buffers there while the other is being added.
        const uint32_t part_bytes = (uint32_t)ti.N * 128u * 4u;
        const bool issuer = warp == kWarpEpi0 && lane == 0;
        ContribIter ci{blockIdx.x + 1}, cc{blockIdx.x + 1};
        uint64_t ib2 = ci.next(W, G, tile_end);
        uint32_t jn = 0;  // next (contributor, operand) job to copy
        auto issue_next = [&]() -> bool {
          if (ib2 >= G) return true;
          const uint32_t b = jn & 1;
          if (jn >= 2 && !mbar_wait(&mg_empty[b], ((jn - 2) >> 1) & 1, abort_s, p.status)) return false;
          mbar_arrive_expect_tx(&mg_full[b], part_bytes);
          bulk_load_g2s(smem + b * kMergeBuf, p.sk_ws + ib2 * slot_floats + (uint64_t)(jn & 1) * p.d_cols * 128,
                        part_bytes, &mg_full[b]);
          if (jn & 1) ib2 = ci.next(W, G, tile_end);
          ++jn;
          return true;
        };
        bool iok = true;
        if (issuer) {
          fence_proxy_async_global();
          fence_proxy_async_smem();
          iok = issue_next() && issue_next();
        }
        uint64_t cb2 = cc.next(W, G, tile_end);
        for (uint32_t j = 0; cb2 < G && ok; ++j) {
          const uint32_t b = j & 1, op = j & 1;
          if (!warp_wait(&mg_full[b], (j >> 1) & 1, abort_s, p.status)) {
            ok = false;
            break;
          }
          const float* sb = reinterpret_cast<const float*>(smem + b * kMergeBuf);
          const uint32_t acc = lane_base + op * (narrow ? acc_cols : 128u);
          // 32 columns per TMEM round trip (N is a multiple of 16).
          for (int n0 = 0; n0 < ti.N; n0 += 32) {
            const bool two = n0 + 16 < ti.N;
            uint32_t v[32];
            tmem_ld_32x32b_x16(acc + n0, *reinterpret_cast<uint32_t(*)[16]>(v));
            if (two) tmem_ld_32x32b_x16(acc + n0 + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
            tmem_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 16; ++jj)
              v[jj] = __float_as_uint(__fadd_rn(__uint_as_float(v[jj]), sb[(n0 + jj) * 128 + m]));
            tmem_st_32x32b_x16(acc + n0, v);
            if (two) {
#pragma unroll
              for (int jj = 16; jj < 32; ++jj)
                v[jj] = __float_as_uint(__fadd_rn(__uint_as_float(v[jj]), sb[(n0 + jj) * 128 + m]));
              tmem_st_32x32b_x16(acc + n0 + 16, v + 16);
            }
          }
          tmem_wait_st();
          __syncwarp();
          if (lane == 0) mbar_arrive(&mg_empty[b]);
          if (issuer && iok) iok = issue_next();
          if (op == 1) cb2 = cc.next(W, G, tile_end);
        }
        ok = ok && __shfl_sync(0xffffffffu, iok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
      for (int n0 = 0; n0 < ti.N; n0 += 8) {
        uint32_t g[8], u[8];
        if (narrow) {
          // Operand sums over the two K halves: (gate, K half 0) at 0,
          // (up, 0) at acc_cols, (gate, 1) at 2 acc_cols, (up, 1) at 3.
          uint32_t g1[8], u1[8];
          tmem_ld_32x32b_x8(lane_base + n0, g);
          tmem_ld_32x32b_x8(lane_base + acc_cols + n0, u);
          tmem_ld_32x32b_x8(lane_base + 2 * acc_cols + n0, g1);
          tmem_ld_32x32b_x8(lane_base + 3 * acc_cols + n0, u1);
          tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            g[jj] = __float_as_uint(__fadd_rn(__uint_as_float(g[jj]), __uint_as_float(g1[jj])));
            u[jj] = __float_as_uint(__fadd_rn(__uint_as_float(u[jj]), __uint_as_float(u1[jj])));
          }
        } else {
          tmem_ld_32x32b_x8(lane_base + n0, g);
          tmem_ld_32x32b_x8(lane_base + 128 + n0, u);
          tmem_wait_ld();
        }
        if (part) {
          // [operand][column][row] so a warp's 32 rows store 128 bytes.
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            my_slot[(uint64_t)(n0 + jj) * 128 + m] = __uint_as_float(g[jj]);
            my_slot[(uint64_t)(p.d_cols + n0 + jj) * 128 + m] = __uint_as_float(u[jj]);
          }
          continue;
        }
        if (p.swiglu) {
          // When the down projection decodes NF4, h is stored in its K order:
          // element 8i+r sits at 8i + 2(r%4) + r/4.
          const int c0 = ti.m_idx * 128 + m;
          const int col = p.h_pair_perm ? ((c0 & ~7) | ((c0 & 3) << 1) | ((c0 >> 2) & 1)) : c0;
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            if (n0 + jj < ti.nv) {
              const float gv = __uint_as_float(g[jj]), uv = __uint_as_float(u[jj]);
              const float hv = __fdividef(gv, 1.0f + __expf(-gv)) * uv;
              const __nv_bfloat16 hb = __float2bfloat16_rn(hv);
              p.h_out[(uint64_t)(ti.pos0 + n0 + jj) * p.ld_out + col] = *reinterpret_cast<const uint16_t*>(&hb);
            }
          }
        } else {
          const int col = ti.m_idx * 256 + m;
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            if (n0 + jj < ti.nv) {
              float* yrow = p.y_out + (uint64_t)(ti.pos0 + n0 + jj) * p.ld_out;
              yrow[col] = __uint_as_float(g[jj]);
              yrow[col + 128] = __uint_as_float(u[jj]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(d_empty);
      ++tit;
      if (part) {
        // Publish this warp's rows: the owner waits for all four warps.
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(p.sk_flags + blockIdx.x, 1);
      }
      if (owner) {
        // Release the partials read: the last of the four reader warps
        // returns each counter to zero for the next launch.
        for (uint64_t b2 = blockIdx.x + 1; b2 < G; ++b2) {
          const uint64_t s0 = W * b2 / G;
          if (s0 >= tile_end) break;
          if (W * (b2 + 1) / G == s0) continue;
          if (lane == 0 && atomicAdd(p.sk_flags + b2, 1) == 2 * kEpiWarps - 1) atomicExch(p.sk_flags + b2, 0);
        }
      }
    }
  }

  __syncthreads();
  if (warp == kWarpMma0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace tc

// Tensor maps of a launch's weights: the packed codes (128 rows x 128 bytes
// per box, 128-byte swizzle) and, for NF4, the scales and zero points
// viewed as [rows, K/64] float32 (K % 256 == 0 keeps the 16-byte row
// stride; a stage reads a 4-block x 128-row box). For 8-bit weights the
// parameter maps are copies of the code map and are not used.
static bool encode_weight_maps(const TcGemmArgs& a, CUtensorMap* raw, CUtensorMap* scl, CUtensorMap* zer) {
  const bool nf4 = a.w.qtype == RIALLM_COMPRESSION_FOUR_BIT;
  const uint64_t row_bytes = nf4 ? (uint64_t)a.K / 2 : (uint64_t)a.K;
  const uint64_t total_rows = (uint64_t)a.E * a.rows_per_expert;
  if (encode_tensor_map_2d(raw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w.data, row_bytes, total_rows,
                           row_bytes, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
    return false;
  if (!nf4) {
    *scl = *raw;
    *zer = *raw;
    return true;
  }
  const uint64_t bpr = (uint64_t)a.K / 64;
  return encode_tensor_map_2d(scl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.w.scales, bpr, total_rows, bpr * 4, 4,
                              128, CU_TENSOR_MAP_SWIZZLE_NONE) == CUDA_SUCCESS &&
         encode_tensor_map_2d(zer, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.w.zero_points, bpr, total_rows, bpr * 4,
                              4, 128, CU_TENSOR_MAP_SWIZZLE_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_tc_gemm(const TcGemmArgs& a, int num_sms, cudaStream_t stream) {
  if (a.P == 0) return cudaSuccess;
  const bool nf4 = a.w.qtype == RIALLM_COMPRESSION_FOUR_BIT;
  CUtensorMap tm_raw, tm_scl, tm_zer, tm_b[4];
  if (!encode_weight_maps(a, &tm_raw, &tm_scl, &tm_zer)) return cudaErrorInvalidValue;
  // The next launch's weights, prefetched at this launch's tail when they
  // have the same format (the kernel variant is per format) and tiles are
  // decode-sized (<= 64 pairs), where a launch's start-up latency is a
  // visible share of its time.
  const TcGemmArgs* nx = a.next;
  const bool pf = nx != nullptr && nx->w.qtype == a.w.qtype && nx->E == a.E && nx->P == a.P &&
                  nx->counts == a.counts && a.max_pairs_per_expert <= 64;
  CUtensorMap tm_nraw = tm_raw, tm_nscl = tm_scl, tm_nzer = tm_zer;
  if (pf && !encode_weight_maps(*nx, &tm_nraw, &tm_nscl, &tm_nzer)) return cudaErrorInvalidValue;
  const uint32_t Ns[4] = {16, 32, 64, 128};
  for (int i = 0; i < 4; ++i)
    if (encode_tensor_map_2d(&tm_b[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.b, (uint64_t)a.K,
                             (uint64_t)a.P, (uint64_t)a.K * 2, 64, Ns[i],
                             CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  // Member by member: a positional initializer would silently shift
  // values when a field is added.
  tc::Params p{};
  p.scales = a.w.scales;
  p.zeros = a.w.zero_points;
  p.n_scales = a.w.n_scales;
  p.n_zeros = a.w.n_zero_points;
  p.K = a.K;
  p.rows_per_expert = a.rows_per_expert;
  p.a1_offset = a.a1_offset;
  p.m_step = a.m_step;
  p.m_tiles = a.m_tiles;
  p.counts = a.counts;
  p.offsets = a.offsets;
  p.E = a.E;
  p.swiglu = a.swiglu ? 1 : 0;
  p.h_pair_perm = a.h_pair_perm ? 1 : 0;
  p.h_out = a.h_out;
  p.y_out = a.y_out;
  p.ld_out = a.ld_out;
  p.status = a.status;
  p.d_cols = a.max_pairs_per_expert <= 64 ? 64 : 128;
  p.sk_ws = a.sk_ws;
  p.sk_flags = a.sk_flags;
  p.flag_wait_ns = a.flag_wait_ns ? a.flag_wait_ns : kWaitLimitNs;
  p.flag_extra = a.flag_extra;
  p.pf_K = pf ? nx->K : 0;
  p.pf_rows_per_expert = pf ? nx->rows_per_expert : 0;
  p.pf_a1_offset = pf ? nx->a1_offset : 0;
  p.pf_m_step = pf ? nx->m_step : 0;
  p.pf_m_tiles = pf ? nx->m_tiles : 0;
  p.pf_sk = pf && nx->sk_ws != nullptr ? 1 : 0;
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
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(tc::kThreads);
  cfg.dynamicSmemBytes = tc::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kern, tm_raw, tm_scl, tm_zer, tm_b[0], tm_b[1], tm_b[2], tm_b[3], tm_nraw,
                                       tm_nscl, tm_nzer, p);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

}  // namespace rl
