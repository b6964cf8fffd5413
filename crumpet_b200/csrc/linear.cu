// crumpet_b200: the Linear projections of a window-attention block (MONAI
// WindowAttention's qkv and proj Linears, which the reference's patched forward
// calls around the attention kernel: torch-ext/crumpet/monai_patch.py:154-197)
// as a tcgen05 GEMM with the bias add fused into the epilogue:
//
//   out[m, n] = sum_k x[m, k] * w[n, k] + bias[n]
//   x [M, K], w [N, K] (nn.Linear layout), out [M, N]; fp16 or bf16, fp32
//   accumulation in tensor memory, one rounding to the element type.
//
// The Swin shapes are skinny (K = 48 or 96 channels, N = 48 .. 256 outputs, M up
// to ~10^6 window tokens): HBM-bound, with the tensor core nearly idle.  One
// persistent CTA per SM, warp-specialised:
//   warp 0      TMA producer: the tile's 128 rows of x as K/16 atoms of
//               [128 rows x 32 B] (32-byte swizzle) into a ring of up to 8 stages;
//   warp 1      MMA issuer: K/16 tcgen05.mma (M=128, N, K=16) into one of two
//               TMEM accumulators (columns 0 / 256), commit -> ring slot free +
//               accumulator full;
//   warps 2..9  two epilogue warpgroups, one per accumulator (tiles alternate):
//               tcgen05.ld of the accumulator (warp w reads TMEM lane quarter
//               w % 4 = rows 32 (w % 4) ..), + bias, round, into the group's
//               row-major staging tile, one TMA store per tile.
// w is loaded once per CTA.  Every mbarrier wait is bounded (2 s); on expiry the
// CTA stops issuing, drains what it issued, frees TMEM and records the error.
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace crumpet {

namespace {

using namespace sm100;

__device__ int g_linear_error;

constexpr int kLinThreads = 320;              // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kLinBM = 128;                   // rows per tile: one TMEM lane each
constexpr int kLinMaxStages = 8;
constexpr int kLinAtomBytes = kLinBM * 32;    // one 16-element K atom of a tile
constexpr uint32_t kLinAccCols = 256;         // columns per TMEM accumulator
constexpr int kLinEpiBar = 1;                 // named barriers 1, 2: the two epilogue groups
constexpr size_t kLinSmemCap = 227 * 1024;

struct LinParams {
  const float* bias;  // [N] (bias values in the element type, widened), or null
  uint32_t N;
  uint32_t tiles;     // ceil(M / 128)
  uint32_t stages;    // ring depth, 2 .. kLinMaxStages
};

struct LinLayout {
  uint32_t w_atom;     // bytes of one K atom of w (N rows x 32 B, 1 KB aligned)
  uint32_t out_tile;   // bytes of one staging tile (128 x N elements)
  uint32_t a_off, w_off, out_off, bias_off, total;
};

__host__ __device__ inline LinLayout lin_layout(int KA, uint32_t N, uint32_t stages) {
  LinLayout l{};
  l.w_atom = (N * 32 + 1023) & ~1023u;
  l.out_tile = kLinBM * N * 2;
  l.a_off = 0;
  l.w_off = l.a_off + stages * KA * kLinAtomBytes;
  l.out_off = l.w_off + KA * l.w_atom;
  l.bias_off = l.out_off + 2 * l.out_tile;
  l.total = l.bias_off + N * 4;
  return l;
}

template <bool BF16>
__device__ __forceinline__ uint32_t lin_pack2(float lo, float hi) {
  if constexpr (BF16) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

__device__ __forceinline__ void lin_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Bounded wait without the abort shortcut, for the shutdown drains.
__device__ __forceinline__ void lin_drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
}

template <int KA, bool BF16>
__global__ void __launch_bounds__(kLinThreads, 1)
    window_linear_kernel(const __grid_constant__ CUtensorMap tx,
                         const __grid_constant__ CUtensorMap tw,
                         const __grid_constant__ CUtensorMap tout, const LinParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ uint64_t full[kLinMaxStages], empty[kLinMaxStages], dfull[2], dempty[2];
  __shared__ uint64_t w_ready, mma_drain;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s, tile_ok_s[2];
  volatile int* abort_flag = &abort_s;

  const uint32_t N = p.N, S = p.stages;
  const LinLayout L = lin_layout(KA, N, S);
  uint8_t* a_ring = smem + L.a_off;
  uint8_t* w_s = smem + L.w_off;
  uint8_t* out_s = smem + L.out_off;
  float* bias_s = reinterpret_cast<float*>(smem + L.bias_off);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    abort_s = 0;
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&dfull[b], 1);
      mbar_init(&dempty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(&w_ready, 1);
    mbar_init(&mma_drain, 1);
    fence_mbar_init();
  }
  for (uint32_t i = threadIdx.x; i < N; i += kLinThreads) bias_s[i] = p.bias ? p.bias[i] : 0.f;
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, 2 * kLinAccCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_map(&tx);
      tma_prefetch_map(&tw);
      tma_prefetch_map(&tout);
      mbar_arrive_expect_tx(&w_ready, KA * N * 32);
      for (int k = 0; k < KA; ++k) tma_load_2d(w_s + k * L.w_atom, &tw, &w_ready, 16 * k, 0);
      uint32_t i = 0;
      for (uint32_t t = blockIdx.x; t < p.tiles; t += gridDim.x, ++i) {
        const uint32_t s = i % S;
        if (i >= S && !mbar_wait(&empty[s], ((i / S) - 1) & 1u, abort_flag)) break;
        mbar_arrive_expect_tx(&full[s], KA * kLinAtomBytes);
#pragma unroll
        for (int k = 0; k < KA; ++k)
          tma_load_2d(a_ring + (s * KA + k) * kLinAtomBytes, &tx, &full[s], 16 * k,
                      int(t * kLinBM));
      }
      // every load issued lands before the CTA may exit
      const uint32_t first = i > S ? i - S : 0;
      for (uint32_t j = first; j < i; ++j) lin_drain_wait(&full[j % S], (j / S) & 1u);
      lin_drain_wait(&w_ready, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kLinBM, int(N), BF16, false);
      bool ok = mbar_wait(&w_ready, 0, abort_flag);
      uint32_t i = 0;
      for (uint32_t t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, ++i) {
        const uint32_t s = i % S, b = i & 1u;
        if (!mbar_wait(&full[s], (i / S) & 1u, abort_flag)) break;
        if (i >= 2 && !mbar_wait(&dempty[b], ((i >> 1) - 1) & 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + b * kLinAccCols;
#pragma unroll
        for (int k = 0; k < KA; ++k) {
          const uint64_t ad =
              smem_desc(smem_u32(a_ring + (s * KA + k) * kLinAtomBytes), 16, 256, kLayoutSW32);
          const uint64_t bd = smem_desc(smem_u32(w_s + k * L.w_atom), 16, 256, kLayoutSW32);
          umma_ss(d, ad, bd, idesc, k > 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
        umma_commit(&dfull[b]);
      }
      // every MMA issued completes before TMEM is freed
      umma_commit(&mma_drain);
      lin_drain_wait(&mma_drain, 0);
    }
  } else {
    // --------------------------------------------------------------- epilogue
    // group e (warps 2..5 / 6..9) takes the tiles of accumulator e: i = e, e + 2, ...
    const uint32_t e = uint32_t(warp - 2) / 4u;
    const uint32_t quarter = uint32_t(warp) & 3u;
    const uint32_t row = quarter * 32 + lane;
    const uint32_t lane_off = (quarter * 32) << 16;
    const bool leader = (uint32_t(warp) & 3u) == 2u && lane == 0;  // warp 2 or 6: waits, stores
    const int bar_id = kLinEpiBar + int(e);
    uint8_t* stage_tile = out_s + e * L.out_tile;
    const uint32_t acc = tmem + lane_off + e * kLinAccCols;
    uint32_t i = e;
    for (uint32_t t = blockIdx.x + e * gridDim.x; t < p.tiles; t += 2 * gridDim.x, i += 2) {
      if (leader) {
        tile_ok_s[e] = mbar_wait(&dfull[e], (i >> 1) & 1u, abort_flag) ? 1 : 0;
        bulk_wait_group_read<0>();  // this group's previous store has read its staging tile
      }
      lin_bar_sync(bar_id, 128);  // one decision for the group's four warps
      if (!tile_ok_s[e]) break;
      tc_fence_after();
      uint8_t* st = stage_tile + row * N * 2;
      for (uint32_t c = 0; c < N; c += 32) {
        uint32_t r[32];
        const bool two = c + 32 <= N;
        if (two) {
          tmem_ld32(acc + c, r);
        } else {
          tmem_ld16(acc + c, *reinterpret_cast<uint32_t(*)[16]>(r));
        }
        tmem_wait_ld();
        const uint32_t width = two ? 32u : 16u;
        for (uint32_t h = 0; h < width; h += 16) {
          uint32_t w[8];
#pragma unroll
          for (int q = 0; q < 8; ++q)
            w[q] = lin_pack2<BF16>(__uint_as_float(r[h + 2 * q]) + bias_s[c + h + 2 * q],
                                   __uint_as_float(r[h + 2 * q + 1]) + bias_s[c + h + 2 * q + 1]);
          *reinterpret_cast<uint4*>(st + 2 * (c + h)) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(st + 2 * (c + h) + 16) = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[e]);
      fence_proxy_async_shared();  // staging writes -> TMA (async proxy) reads
      lin_bar_sync(bar_id, 128);
      if (leader) {
        tma_store_2d(&tout, stage_tile, 0, int(t * kLinBM));
        bulk_commit_group();
      }
    }
    if (leader) bulk_wait_group_all();
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicExch(&g_linear_error, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kLinAccCols);
  }
}

typedef CUresult (*LinEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

LinEncodeFn lin_encode_fn() {
  static LinEncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<LinEncodeFn>(ptr);
  });
  return fn;
}

// 2D map over a row-major [rows, cols] matrix with the given box and swizzle.
int lin_map(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t cols,
            uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz, const char* what) {
  LinEncodeFn enc = lin_encode_fn();
  if (!enc) return set_error(kErrCuda, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1u, 1u};
  const CUtensorMapDataType dt =
      dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kErrInvalid, what);
  return kOk;
}

int lin_num_sms() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

template <int KA, bool BF16>
int launch_lin(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& to,
               const LinParams& p, cudaStream_t stream) {
  auto kern = window_linear_kernel<KA, BF16>;
  // + alignment slack; at least 116 KB so two CTAs never share an SM (each holds
  // all 512 TMEM columns)
  size_t smem = size_t(lin_layout(KA, p.N, p.stages).total) + 1024;
  if (smem < 116 * 1024) smem = 116 * 1024;
  if (smem > kLinSmemCap) return set_error(kErrUnsupported, "window_linear tile does not fit");
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(smem));
  if (e != cudaSuccess) return set_cuda_error(e, "window_linear smem attribute");
  const uint32_t sms = uint32_t(lin_num_sms());
  const uint32_t blocks = p.tiles < sms ? p.tiles : sms;
  kern<<<blocks, kLinThreads, smem, stream>>>(tx, tw, to, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "window_linear launch");
  return kOk;
}

}  // namespace

// K = 48: N up to 256; K = 96: N up to 160 (the 4-stage ring of 24 KB tiles, the
// weights and two staging tiles then still fit in 227 KB of shared memory).
bool window_linear_supported(int64_t K, int64_t N) {
  if (N < 16 || N % 16 != 0) return false;
  return (K == 48 && N <= 256) || (K == 96 && N <= 160);
}

int launch_window_linear(void* out, const void* x, const void* w, const float* bias, int dtype,
                         int64_t M, int64_t K, int64_t N, cudaStream_t stream) {
  if (dtype != kF16 && dtype != kBF16)
    return set_error(kErrInvalid, "window_linear takes float16 or bfloat16 operands");
  if (M < 0) return set_error(kErrInvalid, "M must be non-negative");
  if (!window_linear_supported(K, N))
    return set_error(kErrUnsupported,
                     "window_linear supports K = 48 (N <= 256) or 96 (N <= 160), N a multiple "
                     "of 16");
  if (M == 0) return kOk;
  if (M >= (int64_t(1) << 31) - kLinBM) return set_error(kErrInvalid, "M must be below 2^31");
  if (!out || !x || !w) return set_error(kErrInvalid, "null tensor pointer");
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(x) |
       reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(bias)) & 15u)
    return set_error(kErrInvalid, "tensors must be 16-byte aligned");
  CUtensorMap tx, tw, to;
  if (int rc = lin_map(&tx, x, dtype, uint64_t(M), uint64_t(K), 16, kLinBM,
                       CU_TENSOR_MAP_SWIZZLE_32B, "cuTensorMapEncodeTiled rejected x"))
    return rc;
  if (int rc = lin_map(&tw, w, dtype, uint64_t(N), uint64_t(K), 16, uint32_t(N),
                       CU_TENSOR_MAP_SWIZZLE_32B, "cuTensorMapEncodeTiled rejected w"))
    return rc;
  if (int rc = lin_map(&to, out, dtype, uint64_t(M), uint64_t(N), uint32_t(N), kLinBM,
                       CU_TENSOR_MAP_SWIZZLE_NONE, "cuTensorMapEncodeTiled rejected out"))
    return rc;
  LinParams p{};
  p.bias = bias;
  p.N = uint32_t(N);
  p.tiles = uint32_t((M + kLinBM - 1) / kLinBM);
  // the deepest ring that fits next to the weights and the two staging tiles
  const int KA = int(K / 16);
  p.stages = kLinMaxStages;
  while (p.stages > 2 && size_t(lin_layout(KA, p.N, p.stages).total) + 1024 > kLinSmemCap)
    --p.stages;
  const bool bf = dtype == kBF16;
  if (K == 48) return bf ? launch_lin<3, true>(tx, tw, to, p, stream)
                         : launch_lin<3, false>(tx, tw, to, p, stream);
  return bf ? launch_lin<6, true>(tx, tw, to, p, stream)
            : launch_lin<6, false>(tx, tw, to, p, stream);
}

int read_linear_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_linear_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_linear_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace crumpet
