// crumpet_b200: fused 3D Swin window attention for sm_100a (B200).
//
// Computes, per window b and head h (head_dim 16 or 32, N <= 352 tokens),
//   out[b,h] = softmax(q k^T * scale + bias[h] + mask) v
// with fp32 scores and softmax -- the function of the reference Triton kernel
// torch-ext/crumpet/fused_attention.py:48-146 (eager form: MONAI WindowAttention,
// as described in torch-ext/crumpet/monai_patch.py:117-198).
//
// Design (one persistent CTA per SM, 16 warps):
//   * A tile is 128 query rows of one (window, head).  Three independent tile
//     pipelines ("work groups", WG) run per CTA, each with an MMA-issuing warp and
//     4 softmax warps (one thread per query row = one TMEM lane); one TMA warp
//     feeds all three through a 4-stage shared-memory ring.
//   * TMA loads Q (128 rows) and all K, V rows of the (window, head) with 32-byte
//     swizzle; rows past N are zero-filled.  Two address layouts share the
//     kernel: separate q/k/v [B, H, N, 16] tensors, or the packed qkv Linear
//     output [B, N, 3, H, 16].
//   * Keys are processed in chunks of 64.  The MMA warp computes the chunk's
//     scores in TMEM with tcgen05.mma (M=128, K=16, fp32 accumulation) and then
//     adds the relative-position bias on the tensor cores as well: the bias tile
//     of the (head, query tile), stored as elem(bias)/scale in shared memory,
//     multiplied by a 16x16 identity (one exact product per sum).  So S holds
//     q.k + bias/scale; padded key columns carry -30000 and drop out.
//   * Softmax warps pull S into registers, add a dense mask (global loads, read
//     only for windows flagged in `boundary`) or the analytic shifted-window mask
//     (entries whose roll-side codes differ on a "last window" axis become -inf,
//     the exact limit of the reference's -100), take the chunk maximum, and
//     write P = 2^(x - m_ref) (x = S * scale * log2 e) as fp16/bf16 into one of
//     two TMEM P buffers.  m_ref is a lazy row maximum: it moves only when a
//     chunk exceeds it by more than 8 (P <= 2^8), and then O is rescaled in TMEM.
//     The MMA warp accumulates [O | row sum] += P [V | 1] from TMEM, and the
//     epilogue writes O / row sum.
//   * Bias source: a dense [H, N, N] tensor, or gathered in-kernel from MONAI's
//     relative-position table [T, H] and index [Nc, Nc] (sliced [:N, :N]).
//   * Work: CTAs are split into groups, one per (head, query-tile) pair, and
//     walk the windows in lock step, so the CTAs that need the same K/V rows
//     (the other query tiles and heads of a window) read them close together
//     in time and hit L2.  Warps whose 32 query rows all lie past N skip the
//     math of a tile (their P rows only feed output rows that are discarded).
// Every wait is bounded (2 s of %globaltimer); on expiry the kernel records an
// error in g_device_error, drains its in-flight copies and MMAs, frees TMEM and
// returns.
#include <atomic>
#include <cstdio>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace crumpet {

__device__ int g_device_error;

namespace {

using namespace sm100;

constexpr int kAtom = 16;     // channels per 32-byte swizzle atom (head_dim 16 = one atom)
constexpr int kBM = 128;      // query rows per tile (UMMA M)
constexpr int kCH = 64;       // key chunk
constexpr int kNumWG = 3;      // independent tile pipelines (softmax warpgroups) per CTA
constexpr int kCtrlWarps = 4;  // warp 0: TMA producer; warps 1..kNumWG: MMA issuers
static_assert(kNumWG + 1 <= kCtrlWarps, "one TMA warp and one MMA warp per WG");
constexpr int kSmThreads = kNumWG * 4 * 32;            // softmax threads (one per TMEM lane)
constexpr int kThreads = kCtrlWarps * 32 + kSmThreads;  // 512
constexpr int kRowBytes = kAtom * 2;  // one atom row: 16 channels of fp16/bf16
constexpr int kBarsPerWG = 9;
constexpr int kSchedWords = 7;  // the CTA's work list in shared memory (store_sched)
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 15.f;  // P = 2^(x - m_ref) stays <= 2^15 (fp16 max 65504)
constexpr float kLog2e = 1.4426950408889634f;
// every kPolyEvery-th pair of exponentials is computed on the FMA pipe (poly_ex2x2); at
// stage 0 (ncu medians against all on the SFU) 1 in 6 shortened the kernel by 1.5 %, 1 in 8
// by 1.1 %, 1 in 4 left it unchanged and 1 in 2 lengthened it by 6 % (0: all on the SFU)
constexpr int kPolyEvery = 6;

// Per (padded key count, head dim) layout.  A head dim of 32 is two 16-channel
// atoms: Q, K and V are loaded as one TMA box per atom into separate regions, QK^T
// takes one MMA per atom, and PV one MMA per atom ([V_0 | 1] then V_1).
template <int NPAD, int HD>
struct Cfg {
  static_assert(NPAD % 32 == 0 && NPAD <= 352, "NPAD must be a multiple of 32, at most 352");
  static_assert(HD == 16 || HD == 32, "head_dim 16 or 32");
  static constexpr int NKH = HD / kAtom;              // channel atoms
  // K / V rows per TMA box: NPAD split into equal boxes of at most 128 rows (multiples of
  // 8 rows, so every box starts on the 32-byte swizzle's 256-byte period)
  static constexpr int KVB = NPAD == 352 ? 88 : NPAD == 224 ? 112 : (NPAD < 128 ? NPAD : 128);
  static constexpr int NKB = NPAD / KVB;
  static_assert(NPAD % KVB == 0 && KVB % 8 == 0 && KVB <= 128, "K/V box rows");
  static constexpr int NCH = (NPAD + kCH - 1) / kCH;  // key chunks
  static constexpr int LAST_W = NPAD - (NCH - 1) * kCH;
  static constexpr int STAGES = HD == 16 ? 4 : 2;     // Q/K/V ring stages (shared memory budget)
  static constexpr int NPB = HD == 16 ? 2 : 1;        // P chunk buffers (TMEM budget)
  static constexpr int Q_ATOM = kBM * kRowBytes;
  static constexpr int KV_ATOM = NPAD * kRowBytes;
  static constexpr int Q_BYTES = NKH * Q_ATOM;
  static constexpr int KV_BYTES = NKH * KV_ATOM;
  static constexpr int STAGE_BYTES = Q_BYTES + 2 * KV_BYTES;
  // Bias tile: UMMA A operand, K-major without swizzle: 8x8 core matrices of
  // 128 bytes; core matrix (row group rg, column group cg) at cg * 2048 + rg * 128.
  static constexpr int BIAS_CG_BYTES = (kBM / 8) * 128;  // 2048
  static constexpr int BIAS_BYTES = (NPAD / 8) * BIAS_CG_BYTES;
  // [16 keys][16] of 1.0: every PV MMA (K = 16 keys) reads its ones columns from this one
  // block (the content is the same for every key, so the swizzle does not matter)
  static constexpr int ONES_BYTES = 16 * kRowBytes;
  // Shifted-window mask on the tensor cores: three query-feature tiles (one per axis,
  // [128 rows x 16], UMMA A operand like the bias tile) and one key-feature tile
  // ([NPAD keys x 16], UMMA B operand, K-major without swizzle).
  static constexpr int MASKA_BYTES = 3 * (kBM / 8) * 128 * 2;
  static constexpr int MASKB_BYTES = (NPAD / 8) * 128 * 2;
  // TMEM columns of one WG: S chunk (64), NPB P chunk buffers (32 packed each),
  // O_0 (16) + row sum (16) [+ O_1 (16) for head dim 32].
  static constexpr int TM_S = 0;
  static constexpr int TM_P = kCH;
  static constexpr int TM_O = kCH + NPB * (kCH / 2);
  static constexpr int O_COLS = 2 * kAtom + (NKH - 1) * kAtom;
  // each WG's block starts on a 32-column boundary
  static constexpr uint32_t TMEM_PER_WG = (TM_O + O_COLS + 31) / 32 * 32;
  static_assert(TMEM_PER_WG * kNumWG <= kTmemCols, "TMEM budget");
  static constexpr int IDENT_BYTES = 512;             // 16x16 identity, UMMA B operand
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + BIAS_BYTES + ONES_BYTES +
                                    IDENT_BYTES + MASKA_BYTES + MASKB_BYTES +
                                    (2 * STAGES + kNumWG * kBarsPerWG + 1) * 8 + 64 + 4 * STAGES +
                                    4 * kSchedWords;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

enum MaskMode : int { kMaskNone = 0, kMaskDense = 1, kMaskAnalytic = 2 };

struct KParams {
  // bias: dense [H, N, N] in the element type, or table [T, H] + index [Nc, Nc]
  const uint16_t* bias;
  const void* table;
  const long long* index;
  long long table_rows;  // index values outside [0, table_rows) are flagged, not read
  const uint8_t* bias_tiles;  // prebuilt bias tiles [H * MT][BIAS_BYTES], or null
  int index_stride;
  int bias_from_table;
  int table_f32;
  // dense mask
  const uint16_t* mask;
  const uint8_t* boundary;
  int mask_windows;
  // analytic mask: windows per axis and window / shift sizes of the token grid
  int nwd, nwh, nww, wsd, wsh, wsw, ssd, ssh, ssw;
  // output
  uint16_t* out;
  long long out_sb, out_sh, out_sn;
  int B, H, N, MT, P;
  float scale;
  // Test hook (crumpet_test_stall_attention): the TMA warp issues no loads, so every
  // consumer wait runs into its time limit and the bounded-wait error path runs.
  int stall_loads;
};

// Work list of one CTA: `pair_count` (head, query-tile) pairs starting at pair_begin
// with stride pair_step; inside each pair the windows lo, lo + win_step, ... below hi
// (pair_windows).  Tile k of the CTA (in that order) goes to WG k % kNumWG.
struct Sched {
  int pair_begin, pair_step, pair_count;
  int win_begin, win_step;   // every pair but the first and last: win_begin .. B - 1
  int first_begin, last_end;  // the first pair starts at first_begin, the last ends at last_end
};

// The CTA keeps its Sched in shared memory (kSchedWords words) and reads it at pair
// boundaries only, so none of it stays live in registers through the tile loops.
__device__ __forceinline__ void store_sched(int* dst, const Sched& s) {
  dst[0] = s.pair_begin;
  dst[1] = s.pair_step;
  dst[2] = s.pair_count;
  dst[3] = s.win_begin;
  dst[4] = s.win_step;
  dst[5] = s.first_begin;
  dst[6] = s.last_end;
}

__device__ __forceinline__ int sched_pairs(const volatile int* s) { return s[2]; }

// pair pi of the CTA: its index and its windows lo, lo + step, ... below hi
__device__ __forceinline__ void pair_windows(const volatile int* s, int pi, int B, int& pair,
                                             int& lo, int& hi, int& step) {
  pair = s[0] + pi * s[1];
  lo = pi == 0 ? s[5] : s[3];
  hi = pi == s[2] - 1 ? s[6] : B;
  step = s[4];
}

// With P <= G pairs, S = G / P CTAs share each pair's windows (window b goes to CTA b % S
// of the pair, so the CTAs of one head's query tiles walk the same windows in step and
// meet its K/V rows in L2).  When the bias tiles are prebuilt (`helpers`), the X = G - P * S
// CTAs left over take the last e windows of every pair, split evenly in pair order.  A
// helper's share spans about P / X + 1 pairs, and each pair it starts costs a bias-tile copy
// and a pipeline refill, counted as 6 tiles, so e is the largest value with
//   P e / X + 6 (P / X + 1) <= (B - e) / S,
// i.e. e = (X B - 6 S (P + X)) / (P S + X): the helpers finish no later than the sharing
// CTAs, which now walk B - e windows.  (A bias tile gathered in the kernel costs several
// times that copy, so without prebuilt tiles the leftover CTAs stay idle.)  With P > G
// each CTA takes whole pairs c, c + G, ...
__device__ __forceinline__ Sched make_sched(int P, int B, bool helpers) {
  const int G = gridDim.x, c = blockIdx.x;
  Sched s{0, 1, 0, 0, 1, 0, B};
  if (P <= G) {
    const int S = G / P, X = G - P * S;
    const int64_t room = int64_t(X) * B - int64_t(6) * S * (P + X);
    const int e = (helpers && room > 0) ? int(room / (int64_t(P) * S + X)) : 0;
    if (c < P * S) {
      s.pair_begin = c / S;
      s.pair_count = 1;
      s.win_step = S;
      s.first_begin = c % S;
      s.last_end = B - e;
    } else if (e > 0) {
      const int64_t items = int64_t(P) * e, j = c - P * S;
      const int t0 = int(j * items / X), t1 = int((j + 1) * items / X);
      if (t1 > t0) {
        s.pair_begin = t0 / e;
        s.pair_count = (t1 - 1) / e - t0 / e + 1;
        s.win_begin = B - e;
        s.first_begin = B - e + t0 % e;
        s.last_end = B - e + (t1 - 1) % e + 1;
      }
    }
  } else {
    s.pair_begin = c;
    s.pair_step = G;
    s.pair_count = (P - c + G - 1) / G;
  }
  return s;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for a pair of scores on the FMA pipe instead of the MUFU unit, so the softmax's
// exponentials are not all queued on the SFU: x is clamped to [-125, +inf) (P stays at most
// 2^15 here; below the clamp an fp16 P rounds to 0, while a bf16 P keeps 2^-125, about 1e-38
// of the row's largest term, where the SFU gives 0), split as x = n + f with
// n the nearest integer (the 1.5 * 2^23 rounding constant) and f in [-0.5, 0.5], 2^f taken
// from a cubic fitted for this kernel (minimax by Lawson-reweighted least squares on
// Chebyshev nodes; relative error below 7.5e-5 on [-0.5, 0.5], under half a 16-bit ulp),
// and n added to the result's exponent field.
__device__ __forceinline__ float2 poly_ex2x2(float2 x) {
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  x = make_float2(fmaxf(x.x, -125.f), fmaxf(x.y, -125.f));
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 n = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
  float2 p = __ffma2_rn(make_float2(0.0551716648f, 0.0551716648f), f,
                        make_float2(0.2426111251f, 0.2426111251f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677f, 0.6932609677f));
  p = __ffma2_rn(p, f, make_float2(0.9999280572f, 0.9999280572f));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if constexpr (BF16) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  } else {
    __half2 h = *reinterpret_cast<const __half2*>(&w);
    return __half22float2(h);
  }
}

template <bool BF16>
__device__ __forceinline__ float to_f32(uint16_t h) {
  if constexpr (BF16) {
    return __uint_as_float(uint32_t(h) << 16);
  } else {
    return __half2float(__ushort_as_half(h));
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <bool BF16>
__device__ __forceinline__ uint16_t f32_to_elem(float v) {
  if constexpr (BF16) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  } else {
    return __half_as_ushort(__float2half_rn(v));
  }
}

__device__ __forceinline__ uint32_t ldg_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Waits until *flag == value (bounded like mbar_wait; false on timeout or abort).
__device__ __forceinline__ bool wait_flag_equals(volatile int* flag, int value,
                                                 volatile int* abort) {
  if (*flag == value) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (*flag == value) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      *abort = 1;
      return false;
    }
  }
}

// Waits on a barrier ignoring the abort flag (used only while draining).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
}

// Roll-side code of token t: bit a set when its local coordinate on axis a is
// at or past ws_a - ss_a (the seam of the cyclic roll inside a last window).
__device__ __forceinline__ uint32_t token_code(const KParams& p, int t) {
  const int lw = t % p.wsw;
  const int t2 = t / p.wsw;
  const int lh = t2 % p.wsh;
  const int ld = t2 / p.wsh;
  return uint32_t(ld >= p.wsd - p.ssd) | (uint32_t(lh >= p.wsh - p.ssh) << 1) |
         (uint32_t(lw >= p.wsw - p.ssw) << 2);
}

// Axes (bit a) on which window b is the last window of a shifted grid: there the roll
// seam splits the window into regions whose tokens must not attend to each other.
__device__ __forceinline__ uint32_t window_last_axes(const KParams& p, int b) {
  const int wi = b % (p.nwd * p.nwh * p.nww);
  const int iw = wi % p.nww, t = wi / p.nww;
  const int ih = t % p.nwh, id = t / p.nwh;
  return uint32_t(p.ssd != 0 && id == p.nwd - 1) | (uint32_t(p.ssh != 0 && ih == p.nwh - 1) << 1) |
         (uint32_t(p.ssw != 0 && iw == p.nww - 1) << 2);
}

// Relative-position bias tile of one (head h, query tile mt) for the bias MMA, written
// to dst (shared or global memory) as the UMMA K-major no-swizzle operand image:
// elem(elem(bias) / scale) -- rounded to the element type first, as the reference's
// .to(dtype) -- at rows < N and columns < N; -30000 in padded key columns (their
// scores drop out of the softmax: 2^(-30000 scale log2 e) is 0); 0 in padded query
// rows.  Core matrix (row group rg, column group cg) at cg * (kBM / 8) * 128 + rg * 128.
// Each item is 8 consecutive columns of one row (one 16-byte core-matrix row); two
// items per thread are in flight.  Threads tid = 0 .. nthreads-1 share the work.
template <int NPAD, bool BF16>
__device__ __forceinline__ void build_bias_tile(const KParams& p, int h, int mt, int tid,
                                                int nthreads, uint8_t* dst) {
  constexpr int BIAS_CG = (kBM / 8) * 128;
  constexpr int kItems = kBM * (NPAD / 8);
  constexpr int kBatch = 2;
  const float inv_scale = 1.f / p.scale;
  const uint16_t pad_val = f32_to_elem<BF16>(-30000.f);
  for (int i0 = tid; i0 < kItems; i0 += kBatch * nthreads) {
    float vals[kBatch][8];
    long long idx[kBatch][8];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int item = i0 + u * nthreads;
      const int r = item % kBM, cg = item / kBM;
      const int grow = mt * kBM + r;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int col = cg * 8 + e;
        const bool in = item < kItems && grow < p.N && col < p.N;
        idx[u][e] = -1;
        vals[u][e] = 0.f;
        if (in) {
          if (p.bias_from_table) {
            // -1 marks "not gathered" below, so a stored -1 is mapped to another
            // out-of-range value to be flagged like any other
            const long long v = p.index[(long long)grow * p.index_stride + col];
            idx[u][e] = v == -1 ? -2 : v;
          } else {
            vals[u][e] = to_f32<BF16>(p.bias[(size_t(h) * p.N + grow) * p.N + col]);
          }
        }
      }
    }
    if (p.bias_from_table) {
      // An index value outside the table would read past it: flag it in the
      // device error word (bit 2) and take the bias as 0 instead.
      bool bad = false;
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (idx[u][e] != -1 && (idx[u][e] < 0 || idx[u][e] >= p.table_rows)) {
            bad = true;
            idx[u][e] = -1;
          }
        }
      }
      if (bad) atomicOr(&g_device_error, 2);
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (idx[u][e] >= 0) {
            vals[u][e] =
                p.table_f32
                    ? static_cast<const float*>(p.table)[idx[u][e] * p.H + h]
                    : to_f32<BF16>(
                          static_cast<const uint16_t*>(p.table)[idx[u][e] * p.H + h]);
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int item = i0 + u * nthreads;
      if (item >= kItems) continue;
      const int r = item % kBM, cg = item / kBM;
      const int grow = mt * kBM + r;
      uint32_t wv[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        uint32_t pair = 0;
#pragma unroll
        for (int z = 0; z < 2; ++z) {
          const int col = cg * 8 + e + z;
          uint16_t v16;
          if (grow >= p.N) v16 = 0;
          else if (col >= p.N) v16 = pad_val;
          else v16 = f32_to_elem<BF16>(to_f32<BF16>(f32_to_elem<BF16>(vals[u][e + z])) * inv_scale);
          pair |= uint32_t(v16) << (16 * z);
        }
        wv[e / 2] = pair;
      }
      *reinterpret_cast<uint4*>(dst + cg * BIAS_CG + 16 * r) =
          make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
  }

}

template <int NPAD, int HD, bool BF16, int MASK>
__global__ void __launch_bounds__(kThreads, 1)
window_attention_kernel(const __grid_constant__ CUtensorMap tq,
                        const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const KParams p) {
  using C = Cfg<NPAD, HD>;
  constexpr int kStages = C::STAGES;
  constexpr uint32_t kTmemPerWG = C::TMEM_PER_WG;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint16_t* ones_s = reinterpret_cast<uint16_t*>(smem + kStages * C::STAGE_BYTES);
  uint8_t* bias_s = reinterpret_cast<uint8_t*>(ones_s) + C::ONES_BYTES;
  uint16_t* ident_s = reinterpret_cast<uint16_t*>(bias_s + C::BIAS_BYTES);
  uint8_t* maska_s = reinterpret_cast<uint8_t*>(ident_s) + C::IDENT_BYTES;
  uint8_t* maskb_s = maska_s + C::MASKA_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(maskb_s + C::MASKB_BYTES);
  uint64_t* bias_ready = bars + 2 * kStages + kNumWG * kBarsPerWG;  // one phase per pair
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bias_ready + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Tile index each ring stage was last issued for.  The stages are shared by the
  // warpgroups, so a consumer can reach tile k while the stage's barrier is still
  // two phases behind (its parity then matches an old phase): it first waits for
  // the TMA warp to announce tile k in this word, which implies the previous
  // phase has completed, and only then waits on the barrier's parity.
  volatile int* stage_tile = abort_flag + 1;
  volatile int* sched_s = stage_tile + kStages;  // this CTA's Sched (store_sched)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  {
    const Sched sc = make_sched(p.P, p.B, p.bias_tiles != nullptr);
    if (sc.pair_count == 0) return;  // uniform for the CTA
    if (threadIdx.x == 0) store_sched(const_cast<int*>(sched_s), sc);
  }

  // Barriers: the stage ring [load_full x kStages][load_empty x kStages], then per WG
  //           [s_full][s_empty][p_full][p_empty][o_full][o_empty][drain]
  uint64_t* load_full = bars;
  uint64_t* load_empty = bars + kStages;
  auto bar = [&](int w, int i) { return bars + 2 * kStages + w * kBarsPerWG + i; };
  // kPF/kPE: one barrier per P buffer (kPF + b, kPE + b).  Per-buffer P barriers keep a
  // warp that runs a chunk ahead from arriving on the barrier of the previous chunk.
  constexpr int kSF = 0, kSE = 1, kPF = 2, kPE = 4, kOF = 6, kOE = 7, kDR = 8;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(load_full + s, 1);
      mbar_init(load_empty + s, 1);
    }
    for (int w = 0; w < kNumWG; ++w) {
      mbar_init(bar(w, kSF), 1);
      mbar_init(bar(w, kSE), 4);
      mbar_init(bar(w, kPF), 4);
      mbar_init(bar(w, kPF + 1), 4);
      mbar_init(bar(w, kPE), 1);
      mbar_init(bar(w, kPE + 1), 1);
      mbar_init(bar(w, kOF), 1);
      mbar_init(bar(w, kOE), 4);
      mbar_init(bar(w, kDR), 1);
    }
    mbar_init(bias_ready, 1);
    *abort_flag = 0;
    for (int st = 0; st < kStages; ++st) stage_tile[st] = -1;
    fence_mbar_init();
  }
  if constexpr (MASK == kMaskAnalytic) {
    // Key features of the mask MMA, B[j][2a] = (1 - code_j,a) * pen, B[j][2a+1] = code_j,a * pen
    // with pen = elem(-100 / scale); with the query features A_a[i][2a] = code_i,a,
    // A_a[i][2a+1] = 1 - code_i,a of one axis a, sum_k A_a[i][k] B[j][k] is pen exactly when
    // the two tokens sit on different sides of that axis' roll seam, else 0.  Padded keys
    // get no features (the bias tile already drops them).  K-major without swizzle: element
    // (j, k) at (k / 8) * (NPAD / 8) * 128 + (j / 8) * 128 + (j % 8) * 16 + (k % 8) * 2.
    const uint16_t pen = f32_to_elem<BF16>(-100.f / p.scale);
    uint16_t* mb = reinterpret_cast<uint16_t*>(maskb_s);
    for (int e = threadIdx.x; e < NPAD * 16; e += kThreads) {
      const int j = e >> 4, k = e & 15;
      uint16_t val = 0;
      if (j < p.N && k < 6) {
        const uint32_t bit = (token_code(p, j) >> (k >> 1)) & 1u;
        val = ((k & 1) ? bit : 1u - bit) ? pen : uint16_t(0);
      }
      mb[((k >> 3) * (NPAD / 8) * 128 + (j >> 3) * 128 + (j & 7) * 16 + (k & 7) * 2) / 2] = val;
    }
  }
  {
    // Ones tile: the second 16 columns of the PV B operand, so the MMA also
    // accumulates the row sums of P next to O.
    const uint32_t one2 = BF16 ? 0x3F803F80u : 0x3C003C00u;
    uint32_t* o32 = reinterpret_cast<uint32_t*>(ones_s);
    for (int i = threadIdx.x; i < C::ONES_BYTES / 4; i += kThreads) o32[i] = one2;
    // 16x16 identity (B operand of the bias MMA, K-major, no swizzle: core matrix
    // (n group, k group) at k_group * 256 + n_group * 128, row n at +16 n).
    if (threadIdx.x < 256) {
      const int n = threadIdx.x >> 4, kk = threadIdx.x & 15;
      const uint16_t one = BF16 ? 0x3F80u : 0x3C00u;
      ident_s[((kk >> 3) * 256 + (n >> 3) * 128 + (n & 7) * 16 + (kk & 7) * 2) / 2] =
          n == kk ? one : uint16_t(0);
    }
    fence_proxy_async_shared();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < kCtrlWarps) {
    if (warp == 0) {
      // ------------------------------------------------------------ TMA warp
      // Tiles of the CTA in order k = 0, 1, ...; tile k uses ring stage k % kStages.
      if (lane == 0 && !p.stall_loads) {
        tma_prefetch_map(&tq);
        tma_prefetch_map(&tk);
        tma_prefetch_map(&tv);
        uint32_t k = 0;
        bool ok = true;
        for (int pi = 0; pi < sched_pairs(sched_s) && ok; ++pi) {
          int pair, lo, hi, step;
          pair_windows(sched_s, pi, p.B, pair, lo, hi, step);
          const int h = pair / p.MT, mt = pair - (pair / p.MT) * p.MT;
          for (int b = lo; b < hi && ok; b += step, ++k) {
            const int st = int(k % kStages);
            const uint32_t ph = (k / kStages) & 1u;
            if (!mbar_wait(load_empty + st, ph ^ 1u, abort_flag)) {
              ok = false;
              break;
            }
            uint8_t* sb = smem + st * C::STAGE_BYTES;
            uint64_t* full = load_full + st;
            stage_tile[st] = int(k);
            mbar_arrive_expect_tx(full, C::STAGE_BYTES);
#pragma unroll
            for (int hk = 0; hk < C::NKH; ++hk) {  // one box per 16-channel atom
              tma_load_4d(sb + hk * C::Q_ATOM, &tq, full, kAtom * hk, mt * kBM, h, b);
#pragma unroll
              for (int kb = 0; kb < C::NKB; ++kb) {
                tma_load_4d(sb + C::Q_BYTES + hk * C::KV_ATOM + kb * C::KVB * kRowBytes, &tk, full,
                            kAtom * hk, kb * C::KVB, h, b);
                tma_load_4d(sb + C::Q_BYTES + C::KV_BYTES + hk * C::KV_ATOM + kb * C::KVB * kRowBytes,
                            &tv, full, kAtom * hk, kb * C::KVB, h, b);
              }
            }
          }
        }
        // Drain: every stage's most recent load must have landed before exit.
        for (uint32_t s = 0; s < kStages; ++s) {
          if (k > s) {
            const uint32_t last = ((k - 1 - s) / kStages) * kStages + s;  // last use of stage s
            drain_wait(load_full + int(s), (last / kStages) & 1u);
          }
        }
      }
    } else if (warp <= kNumWG) {
      // ------------------------------------------------------------ MMA warp
      const int w = warp - 1;
      if (lane == 0) {
        const uint32_t tS = tmem_base + w * kTmemPerWG + C::TM_S;
        const uint32_t tP = tmem_base + w * kTmemPerWG + C::TM_P;
        const uint32_t tO = tmem_base + w * kTmemPerWG + C::TM_O;
        const uint32_t ones_addr = smem_u32(ones_s);
        uint32_t it = 0, n_se = 0, n_oe = 0, n_pv = 0;
        bool ok = true;
        auto issue_pv = [&](int c, uint32_t v_addr) -> bool {
          // P chunk n_pv is in buffer n_pv % NPB; its use n_pv / NPB completes that
          // phase of the buffer's P-full barrier
          const uint32_t buf = n_pv % uint32_t(C::NPB);
          if (!mbar_wait(bar(w, kPF + int(buf)), (n_pv / uint32_t(C::NPB)) & 1u, abort_flag))
            return false;
          tc_fence_after();
          if (c == 0) {
            if (!mbar_wait(bar(w, kOE), (n_oe & 1u) ^ 1u, abort_flag)) return false;
            ++n_oe;
            tc_fence_after();
          }
          const int width = (c < C::NCH - 1) ? kCH : C::LAST_W;
          // B = [V_0 | ones]: MN-major, the ones atom sits LBO bytes after this MMA's 16 V
          // rows -- every MMA points at the same 16-row ones block, which lies above the
          // ring -- and further channel atoms V_1.. accumulate into their own 16 columns
          // after the row sums
          constexpr uint32_t idesc_pv = idesc_f16(kBM, 2 * kAtom, BF16, true);
          constexpr uint32_t idesc_pv1 = idesc_f16(kBM, kAtom, BF16, true);
          for (int k = 0; k < width / 16; ++k) {
            const uint32_t pa = tP + buf * uint32_t(kCH / 2) + uint32_t(k * 8);
            const uint32_t acc = (c > 0 || k > 0) ? 1u : 0u;
            const uint32_t row_off = uint32_t(c * kCH + k * 16) * kRowBytes;
            const uint32_t lbo = ones_addr - (v_addr + row_off);
            umma_ts(tO, pa, smem_desc(v_addr + row_off, lbo, 256, kLayoutSW32), idesc_pv, acc);
#pragma unroll
            for (int hk = 1; hk < C::NKH; ++hk) {
              umma_ts(tO + uint32_t(2 * kAtom + (hk - 1) * kAtom), pa,
                      smem_desc(v_addr + hk * C::KV_ATOM + row_off, 16, 256, kLayoutSW32),
                      idesc_pv1, acc);
            }
          }
          umma_commit(bar(w, kPE + int(buf)));
          ++n_pv;
          return true;
        };
        // Bias MMA: S[:, 16i..16i+16) += bias_tile[:, 16i..16i+16) * I16, which adds
        // the (bias / scale) tile to the scores exactly (one non-zero product per sum).
        const uint32_t bias_addr = smem_u32(bias_s);
        const uint32_t maska_addr = smem_u32(maska_s);
        const uint32_t maskb_addr = smem_u32(maskb_s);
        (void)maska_addr;
        (void)maskb_addr;
        const uint64_t ident_desc = smem_desc(smem_u32(ident_s), 256, 128, kLayoutNone);
        constexpr uint32_t idesc_bias = idesc_f16(kBM, 16, BF16, false);
        uint32_t k = 0;
        for (int pi = 0; pi < sched_pairs(sched_s) && ok; ++pi) {
          if (!mbar_wait(bias_ready, uint32_t(pi) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          int pair, lo, hi, step;
          pair_windows(sched_s, pi, p.B, pair, lo, hi, step);
          (void)pair;
          for (int b = lo; b < hi && ok; b += step, ++k) {
            if (int(k % kNumWG) != w) continue;
            const int st = int(k % kStages);
            const uint32_t ph = (k / kStages) & 1u;
            if (!wait_flag_equals(stage_tile + st, int(k), abort_flag) ||
                !mbar_wait(load_full + st, ph, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sb = smem_u32(smem + st * C::STAGE_BYTES);
            // axes on which this window is the last one of a shifted grid
            uint32_t am = 0;
            if constexpr (MASK == kMaskAnalytic) {
              am = window_last_axes(p, b);
              // boundary flags, when the caller gives them, switch the mask off for the
              // windows they leave unflagged (as they do for a dense mask)
              if (p.boundary != nullptr && p.boundary[b] == 0) am = 0;
            }
            const uint32_t q_addr = sb;
            const uint32_t k_addr = sb + C::Q_BYTES;
            const uint32_t v_addr = sb + C::Q_BYTES + C::KV_BYTES;

            for (int c = 0; c < C::NCH && ok; ++c) {
              if (!mbar_wait(bar(w, kSE), (n_se & 1u) ^ 1u, abort_flag)) {
                ok = false;
                break;
              }
              ++n_se;
              tc_fence_after();
              const int width = (c < C::NCH - 1) ? kCH : C::LAST_W;
#pragma unroll
              for (int hk = 0; hk < C::NKH; ++hk) {  // QK^T summed over the channel atoms
                const uint64_t qdesc = smem_desc(q_addr + hk * C::Q_ATOM, 16, 256, kLayoutSW32);
                const uint64_t kdesc = smem_desc(
                    k_addr + hk * C::KV_ATOM + uint32_t(c * kCH) * kRowBytes, 16, 256, kLayoutSW32);
                umma_ss(tS, qdesc, kdesc, idesc_f16(kBM, width, BF16, false), hk > 0 ? 1u : 0u);
              }
              for (int i = 0; i < width / 16; ++i) {
                const uint64_t bdesc = smem_desc(
                    bias_addr + uint32_t(c * (kCH / 8) + 2 * i) * C::BIAS_CG_BYTES,
                    C::BIAS_CG_BYTES, 128, kLayoutNone);
                umma_ss(tS + uint32_t(16 * i), bdesc, ident_desc, idesc_bias, 1u);
              }
              if constexpr (MASK == kMaskAnalytic) {
                // shifted-window mask: one MMA per masked axis adds the penalty where the
                // query and key sit on different sides of that axis' roll seam
                const uint64_t kf = smem_desc(maskb_addr + uint32_t(c * kCH / 8) * 128u,
                                              (NPAD / 8) * 128, 128, kLayoutNone);
#pragma unroll
                for (int a = 0; a < 3; ++a) {
                  if ((am >> a) & 1u) {
                    const uint64_t qf = smem_desc(maska_addr + uint32_t(a) * (kBM / 8) * 256u,
                                                  (kBM / 8) * 128, 128, kLayoutNone);
                    umma_ss(tS, qf, kf, idesc_f16(kBM, width, BF16, false), 1u);
                  }
                }
              }
              umma_commit(bar(w, kSF));
              if (c > 0 && !issue_pv(c - 1, v_addr)) ok = false;
            }
            if (ok && !issue_pv(C::NCH - 1, v_addr)) ok = false;
            if (!ok) break;
            umma_commit(bar(w, kOF));
            umma_commit(load_empty + st);
            ++it;
          }
        }
        // Drain: all MMAs issued by this thread complete before TMEM is freed.
        umma_commit(bar(w, kDR));
        drain_wait(bar(w, kDR), 0);
      }
    }
  } else {
    // -------------------------------------------------------- softmax warps
    const int sw = warp - kCtrlWarps;  // 0 .. 4*kNumWG-1
    const int w = sw >> 2;
    const int quarter = warp & 3;      // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const int tid_sm = threadIdx.x - kCtrlWarps * 32;
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + w * kTmemPerWG + C::TM_S;
    const uint32_t tP = tmem_base + lane_off + w * kTmemPerWG + C::TM_P;
    const uint32_t tO = tmem_base + lane_off + w * kTmemPerWG + C::TM_O;
    const float kNegInf = __int_as_float(0xff800000);
    // S holds q.k + bias/scale; the log2-domain score is x = (S + mask/scale) * scale * log2(e)
    const float2 c1 = make_float2(p.scale * kLog2e, p.scale * kLog2e);
    uint32_t n_sf = 0, n_of = 0;
    uint32_t n_chunk = 0;  // chunks of this WG so far: P buffer n_chunk & 1, its use n_chunk >> 1
    uint32_t k_tile = 0;  // tile index within the CTA (shared numbering with the TMA/MMA warps)
    bool ok = true;

    const int npairs = sched_pairs(sched_s);
    for (int pi = 0; pi < npairs; ++pi) {
      int pair, lo, hi, step;
      pair_windows(sched_s, pi, p.B, pair, lo, hi, step);
      const int h = pair / p.MT, mt = pair - (pair / p.MT) * p.MT;
      // Relative-position bias tile of this (head, query tile) for the bias MMA: copied
      // from prebuilt tiles when the caller has them, else gathered here.
      named_bar_sync(1, kSmThreads);
      if (p.bias_tiles != nullptr) {
        // the tile was built once for this module (attention_bias_tiles): copy it
        const uint4* src = reinterpret_cast<const uint4*>(
            p.bias_tiles + size_t(pair) * size_t(C::BIAS_BYTES));
        uint4* dst = reinterpret_cast<uint4*>(bias_s);
#pragma unroll 4
        for (int i = tid_sm; i < C::BIAS_BYTES / 16; i += kSmThreads) dst[i] = ldg_stream(src + i);
      } else {
        build_bias_tile<NPAD, BF16>(p, h, mt, tid_sm, kSmThreads, bias_s);
      }
      if constexpr (MASK == kMaskAnalytic) {
        // Query features of the mask MMA for this query tile, one [128 x 16] tile per axis a:
        // A_a[r][2a] = code_a(row), A_a[r][2a + 1] = 1 - code_a(row), 0 elsewhere and in rows
        // past N; same core-matrix layout as the bias tile.
        const uint16_t one = BF16 ? 0x3F80u : 0x3C00u;
        uint16_t* ma = reinterpret_cast<uint16_t*>(maska_s);
        for (int e = tid_sm; e < 3 * kBM * 16; e += kSmThreads) {
          const int a = e / (kBM * 16), r = (e / 16) % kBM, k = e % 16;
          const int grow = mt * kBM + r;
          uint16_t val = 0;
          if (grow < p.N && (k >> 1) == a) {
            const uint32_t bit = (token_code(p, grow) >> a) & 1u;
            val = ((k & 1) ? 1u - bit : bit) ? one : uint16_t(0);
          }
          ma[(a * (kBM / 8) * 256 + (k >> 3) * (kBM / 8) * 128 + (r >> 3) * 128 + (r & 7) * 16 +
              (k & 7) * 2) / 2] = val;
        }
      }
      fence_proxy_async_shared();  // bias / mask tiles -> tensor-core (async proxy) reads
      named_bar_sync(1, kSmThreads);
      if (tid_sm == 0) mbar_arrive(bias_ready);
      if (!ok) continue;

      const int qrow = mt * kBM + row;
      const bool valid = qrow < p.N;
      const bool warp_live = (mt * kBM + quarter * 32) < p.N;  // uniform per warp

      for (int b = lo; b < hi && ok; b += step, ++k_tile) {
        if (int(k_tile % kNumWG) != w) continue;
        // ---- per-tile mask state
        bool use_dense = false;
        const uint16_t* mrow = nullptr;
        if constexpr (MASK == kMaskDense) {
          use_dense = (p.boundary == nullptr) || (p.boundary[b] != 0);
          const int mw = b % p.mask_windows;
          mrow = p.mask + (size_t(mw) * p.N + (valid ? qrow : 0)) * p.N;
        }
        // Reference maximum of this row (log2 domain).  P = 2^(x - m_ref) is kept
        // <= 2^15: m_ref moves up only when a chunk exceeds it by more than 15, and
        // then the O accumulator (with the row sums) is rescaled in TMEM first.
        float m_ref = kNegInf;

        // One chunk of W keys (W = 64, or the ragged last chunk).
        auto chunk = [&](auto w_tag, auto tail_tag, int c) -> bool {
          constexpr int W = decltype(w_tag)::value;
          constexpr bool kTail = decltype(tail_tag)::value;
          (void)kTail;
          if (!mbar_wait(bar(w, kSF), n_sf & 1u, abort_flag)) return false;
          ++n_sf;
          tc_fence_after();
          // P buffer of this chunk is free once the PV MMA of its previous use
          // (two chunks ago) has completed.
          const uint32_t pbuf = n_chunk % uint32_t(C::NPB);
          const uint32_t puse_parity = ((n_chunk / uint32_t(C::NPB)) & 1u) ^ 1u;
          if (!warp_live) {
            // No valid row in this warp: keep the barrier protocol, skip the math.
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(w, kSE));
            if (!mbar_wait(bar(w, kPE + int(pbuf)), puse_parity, abort_flag)) return false;
            ++n_chunk;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(w, kPF + int(pbuf)));
            return true;
          }
          uint32_t s[W];
          tmem_ld32(tS, s);
          if constexpr (W > 32) tmem_ld32(tS + 32, s + 32);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(w, kSE));

          // v = q.k + bias/scale (the MMA added the bias tile), plus mask/scale for a
          // dense mask; the log2-domain score is x = v * scale * log2(e).
          float v[W];
#pragma unroll
          for (int j = 0; j < W; ++j) v[j] = __uint_as_float(s[j]);
          if constexpr (MASK == kMaskDense) {
            if (use_dense && valid) {
              // mask row slice: aligned 32-bit words, re-paired when the row starts on
              // an odd element (word k holds elements 2k - odd and 2k - odd + 1)
              const int valid_cols = p.N - c * kCH;
              const uintptr_t addr = reinterpret_cast<uintptr_t>(mrow + c * kCH);
              const uint32_t odd = uint32_t(addr >> 1) & 1u;
              const uint32_t* wp = reinterpret_cast<const uint32_t*>(addr & ~uintptr_t(3));
              const uint32_t sel = odd ? 0x5432u : 0x3210u;
              const float2 inv2 = make_float2(1.f / p.scale, 1.f / p.scale);
#pragma unroll
              for (int g = 0; g < W / 16; ++g) {
                uint32_t mw[9];
#pragma unroll
                for (int k = 0; k < 9; ++k) {
                  const int kk = 8 * g + k;
                  if constexpr (kTail) {
                    mw[k] = (2 * kk - int(odd) < valid_cols) ? ldg_u32(wp + kk) : 0u;
                  } else {
                    mw[k] = ldg_u32(wp + kk);
                  }
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                  const int j = 16 * g + 2 * k;
                  const float2 r = __ffma2_rn(unpack2<BF16>(__byte_perm(mw[k], mw[k + 1], sel)),
                                              inv2, make_float2(v[j], v[j + 1]));
                  v[j] = r.x;
                  v[j + 1] = r.y;
                }
              }
            }
          }
          // chunk maximum: eight independent max3 chains, then a 3-level tree
          float mq[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) mq[q] = kNegInf;
#pragma unroll
          for (int j = 0; j < W; j += 2) mq[(j >> 1) & 7] = max3(mq[(j >> 1) & 7], v[j], v[j + 1]);
          const float mv = fmaxf(fmaxf(max3(mq[0], mq[1], mq[2]), max3(mq[3], mq[4], mq[5])),
                                 fmaxf(mq[6], mq[7]));
          const float mc = mv * c1.x;  // chunk maximum in the log2 domain
          const bool need = mc > m_ref + kRescaleLog2;  // m_ref = -inf: any finite mc
          const float new_ref = need ? mc : m_ref;

          const bool rescale = need && (m_ref != kNegInf);  // O holds sums vs the old m_ref
          if (c > 0 && __any_sync(0xffffffffu, rescale)) {
            // O may be rescaled once the PV MMA of the previous chunk has completed.
            const uint32_t prev = n_chunk - 1;
            if (!mbar_wait(bar(w, kPE + int(prev % uint32_t(C::NPB))),
                           (prev / uint32_t(C::NPB)) & 1u, abort_flag))
              return false;
            tc_fence_after();
            const float f = rescale ? fast_ex2(m_ref - new_ref) : 1.f;
            uint32_t o[2 * kAtom];
            tmem_ld32(tO, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 2 * kAtom; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            tmem_st32(tO, o);
            if constexpr (C::NKH > 1) {
              uint32_t o1[kAtom];
              tmem_ld16(tO + 2 * kAtom, o1);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < kAtom; ++i) o1[i] = __float_as_uint(__uint_as_float(o1[i]) * f);
              tmem_st16(tO + 2 * kAtom, o1);
            }
          }
          if (!mbar_wait(bar(w, kPE + int(pbuf)), puse_parity, abort_flag)) return false;
          tc_fence_after();
          m_ref = new_ref;
          const float mb = (m_ref == kNegInf) ? 0.f : m_ref;
          const float2 nmb = make_float2(-mb, -mb);
          uint32_t pk[W / 2];
#pragma unroll
          for (int k = 0; k < W / 2; ++k) {
            const float2 t = __ffma2_rn(make_float2(v[2 * k], v[2 * k + 1]), c1, nmb);
            if (kPolyEvery > 0 && k % kPolyEvery == kPolyEvery - 1) {
              const float2 e = poly_ex2x2(t);  // every kPolyEvery-th pair on the FMA pipe
              pk[k] = pack2<BF16>(e.x, e.y);
            } else {
              pk[k] = pack2<BF16>(fast_ex2(t.x), fast_ex2(t.y));
            }
          }
          const uint32_t tPb = tP + pbuf * uint32_t(kCH / 2);
          tmem_st16(tPb, pk);
          if constexpr (W > 32) tmem_st16(tPb + 16, pk + 16);
          ++n_chunk;
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(w, kPF + int(pbuf)));
          return true;
        };

        for (int c = 0; c < C::NCH - 1 && ok; ++c)
          ok = chunk(std::integral_constant<int, kCH>{}, std::false_type{}, c);
        if (ok) ok = chunk(std::integral_constant<int, C::LAST_W>{}, std::true_type{}, C::NCH - 1);
        if (!ok) break;

        // ---- epilogue: O / row sum
        if (!mbar_wait(bar(w, kOF), n_of & 1u, abort_flag)) {
          ok = false;
          break;
        }
        ++n_of;
        tc_fence_after();
        if (!warp_live) {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(w, kOE));
          continue;
        }
        uint32_t o[2 * kAtom];
        uint32_t o1[kAtom];  // channels 16..31 (head dim 32)
        tmem_ld32(tO, o);
        if constexpr (C::NKH > 1) tmem_ld16(tO + 2 * kAtom, o1);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(w, kOE));
        if (valid) {
          const float inv = 1.f / __uint_as_float(o[kAtom]);  // row sum
          uint16_t* dst = p.out + b * p.out_sb + h * p.out_sh + qrow * p.out_sn;
          uint32_t packed[kAtom / 2];
#pragma unroll
          for (int d = 0; d < kAtom; d += 2)
            packed[d / 2] = pack2<BF16>(__uint_as_float(o[d]) * inv, __uint_as_float(o[d + 1]) * inv);
          stg(reinterpret_cast<uint4*>(dst), make_uint4(packed[0], packed[1], packed[2], packed[3]));
          stg(reinterpret_cast<uint4*>(dst + 8),
              make_uint4(packed[4], packed[5], packed[6], packed[7]));
          if constexpr (C::NKH > 1) {
#pragma unroll
            for (int d = 0; d < kAtom; d += 2)
              packed[d / 2] =
                  pack2<BF16>(__uint_as_float(o1[d]) * inv, __uint_as_float(o1[d + 1]) * inv);
            stg(reinterpret_cast<uint4*>(dst + 16),
                make_uint4(packed[0], packed[1], packed[2], packed[3]));
            stg(reinterpret_cast<uint4*>(dst + 24),
                make_uint4(packed[4], packed[5], packed[6], packed[7]));
          }
        }
      }
    }
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicOr(&g_device_error, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Prebuilt bias tiles: block `pair` (= h * MT + mt) writes the tile the attention kernel
// would gather for that (head, query tile), in the same shared-memory image.
template <int NPAD, bool BF16>
__global__ void __launch_bounds__(256) bias_tile_kernel(const KParams p, uint8_t* tiles) {
  const int pair = blockIdx.x;
  const int h = pair / p.MT, mt = pair - h * p.MT;
  build_bias_tile<NPAD, BF16>(p, h, mt, threadIdx.x, blockDim.x,
                              tiles + size_t(pair) * size_t(Cfg<NPAD, 16>::BIAS_BYTES));
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 4D map {head_dim, N, H, B} over q/k/v: boxes of one 16-channel atom x box_rows rows
// (128 for Q, the K/V box height of the chosen key padding for K and V), 32-byte swizzle.
int make_qkv_map(CUtensorMap* map, const void* base, const AttnArgs& a, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return set_error(kErrCuda, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[4] = {cuuint64_t(a.head_dim), cuuint64_t(a.N), cuuint64_t(a.H),
                              cuuint64_t(a.B)};
  const cuuint64_t strides[3] = {cuuint64_t(a.qkv_stride_n) * 2, cuuint64_t(a.qkv_stride_h) * 2,
                                 cuuint64_t(a.qkv_stride_b) * 2};
  const cuuint32_t box[4] = {cuuint32_t(kAtom), cuuint32_t(box_rows), 1u, 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapDataType dt =
      a.dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kErrInvalid, "cuTensorMapEncodeTiled rejected q/k/v");
  return kOk;
}

int num_sms() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

template <int NPAD, int HD, bool BF16, int MASK>
int launch_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                const KParams& kp, cudaStream_t stream) {
  using C = Cfg<NPAD, HD>;
  auto kern = window_attention_kernel<NPAD, HD, BF16, MASK>;
  static bool configured[64] = {false};  // per device; the attribute is per function
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error(e, "attention smem attribute");
    configured[dev] = true;
  }
  kern<<<num_sms(), kThreads, C::SMEM_BYTES, stream>>>(tq, tk, tv, kp);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "attention launch");
  return kOk;
}

template <int NPAD, int HD>
int dispatch_mode(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk,
                  const CUtensorMap& tv, const KParams& kp, cudaStream_t stream) {
  const int mode = a.analytic ? kMaskAnalytic : (a.mask ? kMaskDense : kMaskNone);
  if (a.dtype == kBF16) {
    if (mode == kMaskDense) return launch_impl<NPAD, HD, true, kMaskDense>(tq, tk, tv, kp, stream);
    if (mode == kMaskAnalytic)
      return launch_impl<NPAD, HD, true, kMaskAnalytic>(tq, tk, tv, kp, stream);
    return launch_impl<NPAD, HD, true, kMaskNone>(tq, tk, tv, kp, stream);
  }
  if (mode == kMaskDense) return launch_impl<NPAD, HD, false, kMaskDense>(tq, tk, tv, kp, stream);
  if (mode == kMaskAnalytic)
    return launch_impl<NPAD, HD, false, kMaskAnalytic>(tq, tk, tv, kp, stream);
  return launch_impl<NPAD, HD, false, kMaskNone>(tq, tk, tv, kp, stream);
}

template <int NPAD>
int dispatch_npad(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk,
                  const CUtensorMap& tv, const KParams& kp, cudaStream_t stream) {
  if (a.head_dim == 32) return dispatch_mode<NPAD, 32>(a, tq, tk, tv, kp, stream);
  return dispatch_mode<NPAD, 16>(a, tq, tk, tv, kp, stream);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

std::atomic<int> g_test_stall{0};

}  // namespace

int set_attention_test_stall(int enable) { return g_test_stall.exchange(enable ? 1 : 0); }

int launch_window_attention(const AttnArgs& a, cudaStream_t stream) {
  if (a.dtype != kF16 && a.dtype != kBF16 && a.dtype != kF32)
    return set_error(kErrUnsupported,
                     "fused_swin_attention supports float32, float16 and bfloat16");
  if (!simt_attention_head_dim(a.head_dim))
    return set_error(kErrUnsupported,
                     "fused_swin_attention requires a power-of-two head_dim between 16 and 256");
  if (a.N < 1) return set_error(kErrUnsupported, "fused_swin_attention requires N >= 1");
  if (a.B < 0 || a.H < 1) return set_error(kErrInvalid, "B must be >= 0 and H >= 1");
  if (!(a.scale > 0.f) || !(a.scale < 1e30f))
    return set_error(kErrUnsupported, "fused_swin_attention requires a finite scale > 0");
  if (a.B == 0) return kOk;
  if (a.B > 0x7fffffff || a.H > 0xffff || a.N > 0xffffff)
    return set_error(kErrInvalid, "B, H or N too large");
  if (!a.q || !a.k || !a.v || !a.out) return set_error(kErrInvalid, "null tensor pointer");
  const bool gather = a.bias_from_table && !a.bias_tiles;
  if (a.bias_tiles ? false : (a.bias_from_table ? (!a.table || !a.index) : !a.bias))
    return set_error(kErrInvalid, "null bias pointer");
  if (a.bias_tiles && (reinterpret_cast<uintptr_t>(a.bias_tiles) & 15u))
    return set_error(kErrInvalid, "bias tiles must be 16-byte aligned");
  if (gather && a.index_stride < a.N)
    return set_error(kErrInvalid, "relative position index is smaller than N x N");
  if (gather && a.table_rows < 1)
    return set_error(kErrInvalid, "relative position bias table has no rows");
  if (a.mask && a.mask_windows < 1) return set_error(kErrInvalid, "mask_windows must be >= 1");
  if (a.analytic) {
    if (a.mask) return set_error(kErrInvalid, "analytic and dense masks are exclusive");
    if (a.win[0] * a.win[1] * a.win[2] != a.N || a.nwin[0] < 1 || a.nwin[1] < 1 || a.nwin[2] < 1)
      return set_error(kErrInvalid, "analytic mask geometry does not match N");
    for (int i = 0; i < 3; ++i)
      if (a.shift[i] < 0 || a.shift[i] >= a.win[i])
        return set_error(kErrInvalid, "analytic mask shift must satisfy 0 <= shift < window");
  }
  // The tensor-core kernel: fp16 / bf16, head_dim 16 or 32, N <= 352, q/k/v/out on
  // 16-byte boundaries with 16-byte row strides (TMA); everything else runs the
  // fp32 SIMT kernel (attention_simt.cu).
  const bool tensor_path =
      a.dtype != kF32 && (a.head_dim == 16 || a.head_dim == 32) && a.N <= 352 &&
      aligned16(a.q) && aligned16(a.k) && aligned16(a.v) && aligned16(a.out) &&
      (a.qkv_stride_n | a.qkv_stride_h | a.qkv_stride_b) % 8 == 0 &&
      (a.out_stride_n | a.out_stride_h | a.out_stride_b) % 8 == 0;
  if (!tensor_path) {
    if (a.bias_tiles)
      return set_error(kErrUnsupported,
                       "prebuilt bias tiles apply to fp16 / bf16 head_dim 16 or 32 windows of at "
                       "most 352 tokens with 16-byte aligned tensors");
    return launch_window_attention_simt(a, stream);
  }

  const int n32 = int((a.N + 31) / 32) * 32;
  const int npad = n32 <= 64 ? 64 : n32 <= 128 ? 128 : n32 <= 224 ? 224 : 352;
  int kv_rows = 128;
  switch (npad) {
    case 64: kv_rows = Cfg<64, 16>::KVB; break;
    case 128: kv_rows = Cfg<128, 16>::KVB; break;
    case 224: kv_rows = Cfg<224, 16>::KVB; break;
    default: kv_rows = Cfg<352, 16>::KVB; break;
  }
  CUtensorMap tq, tk, tv;
  if (int e = make_qkv_map(&tq, a.q, a, kBM)) return e;
  if (int e = make_qkv_map(&tk, a.k, a, kv_rows)) return e;
  if (int e = make_qkv_map(&tv, a.v, a, kv_rows)) return e;

  KParams kp{};
  kp.bias = static_cast<const uint16_t*>(a.bias);
  kp.table = a.table;
  kp.index = reinterpret_cast<const long long*>(a.index);
  kp.index_stride = int(a.index_stride);
  kp.table_rows = a.table_rows;
  kp.bias_tiles = static_cast<const uint8_t*>(a.bias_tiles);
  kp.bias_from_table = a.bias_from_table ? 1 : 0;
  kp.table_f32 = a.table_f32 ? 1 : 0;
  kp.mask = static_cast<const uint16_t*>(a.mask);
  kp.boundary = a.boundary;
  kp.mask_windows = a.mask ? int(a.mask_windows) : 1;
  kp.nwd = int(a.nwin[0]);
  kp.nwh = int(a.nwin[1]);
  kp.nww = int(a.nwin[2]);
  kp.wsd = int(a.win[0]);
  kp.wsh = int(a.win[1]);
  kp.wsw = int(a.win[2]);
  kp.ssd = int(a.shift[0]);
  kp.ssh = int(a.shift[1]);
  kp.ssw = int(a.shift[2]);
  kp.out = static_cast<uint16_t*>(a.out);
  kp.out_sb = a.out_stride_b;
  kp.out_sh = a.out_stride_h;
  kp.out_sn = a.out_stride_n;
  kp.B = int(a.B);
  kp.H = int(a.H);
  kp.N = int(a.N);
  kp.MT = int((a.N + kBM - 1) / kBM);
  kp.P = kp.H * kp.MT;
  kp.scale = a.scale;
  kp.stall_loads = g_test_stall.load(std::memory_order_relaxed);
  if (!a.analytic) {
    // keep the analytic-mask geometry harmless when unused
    kp.nwd = kp.nwh = kp.nww = 1;
    kp.wsd = kp.wsh = kp.wsw = 1;
  }

  if (n32 <= 64) return dispatch_npad<64>(a, tq, tk, tv, kp, stream);
  if (n32 <= 128) return dispatch_npad<128>(a, tq, tk, tv, kp, stream);
  if (n32 <= 224) return dispatch_npad<224>(a, tq, tk, tv, kp, stream);
  return dispatch_npad<352>(a, tq, tk, tv, kp, stream);
}

namespace {
int npad_for(int64_t N) {
  const int64_t n32 = (N + 31) / 32 * 32;
  return n32 <= 64 ? 64 : n32 <= 128 ? 128 : n32 <= 224 ? 224 : 352;
}
// one (head, query tile) tile: NPAD / 8 column groups of kBM / 8 core matrices of 8 x 8
// 16-bit elements (128 bytes) -- Cfg<NPAD, HD>::BIAS_BYTES, the stride the kernels use
int64_t bias_tile_bytes(int npad) { return int64_t(npad / 8) * (kBM / 8) * 128; }
template <int NPAD>
int launch_bias_tiles_npad(uint8_t* tiles, const KParams& kp, int dtype, cudaStream_t stream) {
  if (dtype == kBF16)
    bias_tile_kernel<NPAD, true><<<kp.P, 256, 0, stream>>>(kp, tiles);
  else
    bias_tile_kernel<NPAD, false><<<kp.P, 256, 0, stream>>>(kp, tiles);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "bias tile launch");
  return kOk;
}
}  // namespace

static_assert(Cfg<352, 16>::BIAS_BYTES == (352 / 8) * (kBM / 8) * 128 &&
                  Cfg<224, 16>::BIAS_BYTES == (224 / 8) * (kBM / 8) * 128,
              "bias tile size on the host and in the kernels");

int64_t attention_bias_tiles_bytes(int64_t H, int64_t N) {
  if (H < 1 || N < 1 || N > 352) return 0;
  return H * ((N + kBM - 1) / kBM) * bias_tile_bytes(npad_for(N));
}

int launch_attention_bias_tiles(void* tiles, const AttnArgs& a, cudaStream_t stream) {
  if (a.dtype != kF16 && a.dtype != kBF16)
    return set_error(kErrUnsupported, "bias tiles are built for float16 or bfloat16");
  if (a.N < 1 || a.N > 352 || a.H < 1 || a.H > 0xffff)
    return set_error(kErrUnsupported, "bias tiles need 1 <= N <= 352 and 1 <= H");
  if (!(a.scale > 0.f) || !(a.scale < 1e30f))
    return set_error(kErrUnsupported, "bias tiles need a finite scale > 0");
  if (!tiles || !a.table || !a.index) return set_error(kErrInvalid, "null tensor pointer");
  if (reinterpret_cast<uintptr_t>(tiles) & 15u)
    return set_error(kErrInvalid, "bias tiles must be 16-byte aligned");
  if (a.index_stride < a.N) return set_error(kErrInvalid, "relative position index is smaller than N x N");
  if (a.table_rows < 1) return set_error(kErrInvalid, "relative position bias table has no rows");
  KParams kp{};
  kp.table = a.table;
  kp.table_f32 = a.table_f32 ? 1 : 0;
  kp.table_rows = a.table_rows;
  kp.index = reinterpret_cast<const long long*>(a.index);
  kp.index_stride = int(a.index_stride);
  kp.bias_from_table = 1;
  kp.H = int(a.H);
  kp.N = int(a.N);
  kp.MT = int((a.N + kBM - 1) / kBM);
  kp.P = kp.H * kp.MT;
  kp.scale = a.scale;
  uint8_t* t = static_cast<uint8_t*>(tiles);
  switch (npad_for(a.N)) {
    case 64: return launch_bias_tiles_npad<64>(t, kp, a.dtype, stream);
    case 128: return launch_bias_tiles_npad<128>(t, kp, a.dtype, stream);
    case 224: return launch_bias_tiles_npad<224>(t, kp, a.dtype, stream);
    default: return launch_bias_tiles_npad<352>(t, kp, a.dtype, stream);
  }
}

// ---------------------------------------------------------------------------------
// Bias tiles in a fixed device buffer, for callers that cannot allocate device memory
// (crumpet_swin_window_attention_qkv_static_tiles).  The buffer is part of the library
// image: every GPU that loads the library holds kStaticTileBytes until the process exits.
// Its name is only a host-side stand-in for the device copy, so host code passes the
// device address, looked up once per device with that device current.
constexpr size_t kStaticTileBytes = size_t(4) << 20;
static __device__ __align__(256) uint8_t g_static_bias_tiles[kStaticTileBytes];

namespace {
constexpr int kMaxStaticDevices = 64;

int static_tiles_address(void** out) {
  static std::mutex mu;
  static void* addr[kMaxStaticDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxStaticDevices)
    return set_error(kErrUnsupported, "static bias tiles: device ordinal above 63");
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_bias_tiles);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaGetSymbolAddress(static bias tiles)");
    addr[dev] = p;
  }
  *out = addr[dev];
  return kOk;
}
}  // namespace

int launch_window_attention_static_tiles(const AttnArgs& a, cudaStream_t stream) {
  const int64_t need = attention_bias_tiles_bytes(a.H, a.N);
  if (need <= 0)
    return set_error(kErrUnsupported, "static bias tiles need 1 <= N <= 352 and H >= 1");
  if (uint64_t(need) > kStaticTileBytes)
    return set_error(kErrUnsupported,
                     "static bias tiles: H x ceil(N / 128) tiles exceed the 4 MiB buffer "
                     "(at most 46 tiles at N = 343, 73 at N = 216)");
  void* tiles = nullptr;
  if (int rc = static_tiles_address(&tiles)) return rc;
  // every byte of the `need` bytes the attention kernel reads is rewritten here, so the
  // previous call's contents never show through
  if (int rc = launch_attention_bias_tiles(tiles, a, stream)) return rc;
  AttnArgs t = a;
  t.bias_tiles = tiles;
  return launch_window_attention(t, stream);
}

int read_device_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  }
  const int lin = read_linear_error(clear);  // the Linear kernel's own word
  if (lin < 0) return -1;
  return v | lin;
}

}  // namespace crumpet
