// crumpet_b200: window attention for the inputs the tensor-core kernel does not take.
//
// Same function as attention.cu -- per window b and head h,
//   out[b,h] = softmax(q k^T * scale + bias[h] + mask) v
// (torch-ext/crumpet/fused_attention.py:48-146) -- for float32 q/k/v, head dims
// 64 to 256, and windows of more than 384 tokens, which the reference's Triton
// launcher accepts (any power-of-two head_dim >= 16, any dtype tl.dot takes) and the
// tcgen05 kernel (fp16/bf16, head_dim 16/32, N <= 384) does not.
//
// Design: plain fp32 FMA arithmetic, one CTA of 128 threads per (query block,
// head, window).  A query row belongs to TPR = max(1, D/32) adjacent lanes, each
// holding E = D/TPR channels of q and of the output accumulator in registers;
// the partial dot products are summed with xor-shuffles inside the lane group.
// Keys stream in chunks of 32: the chunk's K and V rows are converted to fp32
// into shared memory (each lane-group slice padded by 4 floats so the slices of
// one row sit in different banks for the 16-byte reads), and the bias tile of the
// CTA's rows x the chunk's keys -- dense [H, N, N], or gathered from MONAI's
// table [T, H] by the relative-position index sliced [:N, :N] -- is staged with the
// mask already added (dense mask rows of flagged windows, or the shifted-window
// mask computed from roll-side codes), read coalesced along the keys.  Online
// softmax per chunk in the log2 domain with exp2f.  Masked entries add -100, as the
// reference's mask does.  No waits, so no bounded-wait error path is needed.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace crumpet {

extern __device__ int g_device_error;

namespace {

constexpr int kThreads = 128;
constexpr int kKC = 32;  // keys per chunk
constexpr float kLog2e = 1.4426950408889634f;

struct SimtParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  long long qs_b, qs_h, qs_n;  // element strides of q / k / v
  long long os_b, os_h, os_n;  // element strides of out
  const void* bias;            // dense [H, N, N] in the element type
  const void* table;           // [T, H]: fp32 (table_f32) or the element type
  const long long* index;      // [>= N, index_stride]
  long long table_rows, index_stride;
  int bias_from_table, table_f32;
  const void* mask;            // dense [mask_windows, N, N] in the element type, or null
  const uint8_t* boundary;     // [B] or null
  int mask_windows;
  int analytic;                // shifted-window mask from the window geometry
  int nwd, nwh, nww, wsd, wsh, wsw, ssd, ssh, ssw;
  int B, H, N, QB;             // QB = query blocks per (window, head)
  float scale;
};

template <typename T>
__device__ __forceinline__ float load_f32(const T* p, long long i);
template <>
__device__ __forceinline__ float load_f32<float>(const float* p, long long i) {
  return __ldg(p + i);
}
template <>
__device__ __forceinline__ float load_f32<__half>(const __half* p, long long i) {
  return __half2float(__ldg(p + i));
}
template <>
__device__ __forceinline__ float load_f32<__nv_bfloat16>(const __nv_bfloat16* p, long long i) {
  return __bfloat162float(__ldg(p + i));
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Roll-side code of token t (bit a: local coordinate on axis a at or past ws - ss);
// two tokens of a window on its last position along a shifted axis carry different
// region labels exactly when their codes differ on that axis.
__device__ __forceinline__ uint32_t side_code(const SimtParams& p, int t) {
  const int lw = t % p.wsw, t2 = t / p.wsw;
  const int lh = t2 % p.wsh, ld = t2 / p.wsh;
  return uint32_t(ld >= p.wsd - p.ssd) | (uint32_t(lh >= p.wsh - p.ssh) << 1) |
         (uint32_t(lw >= p.wsw - p.ssw) << 2);
}

template <int D>
struct Shape {
  static constexpr int TPR = D >= 64 ? D / 32 : 1;  // lanes per query row
  static constexpr int E = D / TPR;                  // channels per lane
  static constexpr int R = kThreads / TPR;           // query rows per CTA
  static constexpr int SLICE = E + (TPR > 1 ? 4 : 0);
  static constexpr int ROW = TPR * SLICE;            // floats per K / V row in shared memory
  static constexpr int TILE = kKC + 1;               // bias tile row (odd: no bank conflicts)
  static constexpr int SMEM = (2 * kKC * ROW + R * TILE) * 4 + kKC * 4;
  static_assert(E % 4 == 0 && E <= 32, "channels per lane");
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) window_attention_simt_kernel(const SimtParams p) {
  using S = Shape<D>;
  extern __shared__ float4 smem4[];
  float* ks = reinterpret_cast<float*>(smem4);
  float* vs = ks + kKC * S::ROW;
  float* tile = vs + kKC * S::ROW;
  uint32_t* key_code = reinterpret_cast<uint32_t*>(tile + S::R * S::TILE);

  const int tid = threadIdx.x;
  const int row = tid / S::TPR;       // query row of this lane inside the block
  const int part = tid % S::TPR;      // channel slice of this lane
  long long blk = blockIdx.x;
  const int qb = int(blk % p.QB);
  blk /= p.QB;
  const int h = int(blk % p.H);
  const int b = int(blk / p.H);
  const int q0 = qb * S::R;
  const int i = q0 + row;
  const bool valid = i < p.N;

  const T* qg = static_cast<const T*>(p.q) + b * p.qs_b + h * p.qs_h;
  const T* kg = static_cast<const T*>(p.k) + b * p.qs_b + h * p.qs_h;
  const T* vg = static_cast<const T*>(p.v) + b * p.qs_b + h * p.qs_h;

  float qr[S::E], acc[S::E];
#pragma unroll
  for (int e = 0; e < S::E; ++e) {
    qr[e] = valid ? load_f32(qg, (long long)i * p.qs_n + part * S::E + e) : 0.f;
    acc[e] = 0.f;
  }
  const float qk_scale = p.scale * kLog2e;
  float m = -INFINITY, l = 0.f;

  // per-window mask state
  const bool dense = p.mask != nullptr && (p.boundary == nullptr || p.boundary[b] != 0);
  const T* mrow_base = dense ? static_cast<const T*>(p.mask) +
                                   (long long)(b % p.mask_windows) * p.N * p.N
                             : nullptr;
  uint32_t last_axes = 0;
  if (p.analytic && (p.boundary == nullptr || p.boundary[b] != 0)) {
    const int wi = b % (p.nwd * p.nwh * p.nww);
    const int iw = wi % p.nww, t = wi / p.nww;
    const int ih = t % p.nwh, id = t / p.nwh;
    last_axes = uint32_t(p.ssd != 0 && id == p.nwd - 1) |
                (uint32_t(p.ssh != 0 && ih == p.nwh - 1) << 1) |
                (uint32_t(p.ssw != 0 && iw == p.nww - 1) << 2);
  }
  bool bad_index = false;

  for (int k0 = 0; k0 < p.N; k0 += kKC) {
    __syncthreads();  // the previous chunk's shared tiles are no longer read
    // K / V rows of the chunk, converted to fp32 (rows past N are zero)
    for (int f = tid; f < kKC * D; f += kThreads) {
      const int j = f / D, d = f % D;
      const int kk = k0 + j;
      const int s = j * S::ROW + (d / S::E) * S::SLICE + d % S::E;
      const bool in = kk < p.N;
      ks[s] = in ? load_f32(kg, (long long)kk * p.qs_n + d) : 0.f;
      vs[s] = in ? load_f32(vg, (long long)kk * p.qs_n + d) : 0.f;
    }
    if (p.analytic && tid < kKC) key_code[tid] = k0 + tid < p.N ? side_code(p, k0 + tid) : 0u;
    if (p.analytic) __syncthreads();
    // bias (+ mask) tile of the block's rows x the chunk's keys, coalesced along keys
    for (int f = tid; f < S::R * kKC; f += kThreads) {
      const int r = f / kKC, j = f % kKC;
      const int gi = q0 + r, kk = k0 + j;
      float val = 0.f;
      if (kk >= p.N) {
        val = -INFINITY;  // padded key: drops out of the softmax
      } else if (gi < p.N) {
        if (p.bias_from_table) {
          long long idx = p.index[(long long)gi * p.index_stride + kk];
          if (idx < 0 || idx >= p.table_rows) {
            bad_index = true;
          } else {
            val = p.table_f32 ? __ldg(static_cast<const float*>(p.table) + idx * p.H + h)
                              : load_f32(static_cast<const T*>(p.table), idx * p.H + h);
            // the reference rounds the gathered bias to the activation dtype
            val = float(from_f32<T>(val));
          }
        } else {
          val = load_f32(static_cast<const T*>(p.bias), ((long long)h * p.N + gi) * p.N + kk);
        }
        if (dense) {
          val += load_f32(mrow_base, (long long)gi * p.N + kk);
        } else if (last_axes != 0) {
          const uint32_t ci = side_code(p, gi);
          if ((ci ^ key_code[j]) & last_axes) val += -100.f;
        }
      }
      tile[r * S::TILE + j] = val;
    }
    __syncthreads();

    // scores of this row against the chunk, log2 domain
    float s[kKC];
    float mc = -INFINITY;
#pragma unroll
    for (int j = 0; j < kKC; ++j) {
      const float4* kr = reinterpret_cast<const float4*>(ks + j * S::ROW + part * S::SLICE);
      float dot = 0.f;
#pragma unroll
      for (int e4 = 0; e4 < S::E / 4; ++e4) {
        const float4 kv = kr[e4];
        dot = fmaf(qr[4 * e4], kv.x, dot);
        dot = fmaf(qr[4 * e4 + 1], kv.y, dot);
        dot = fmaf(qr[4 * e4 + 2], kv.z, dot);
        dot = fmaf(qr[4 * e4 + 3], kv.w, dot);
      }
#pragma unroll
      for (int off = 1; off < S::TPR; off <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      s[j] = fmaf(dot, qk_scale, tile[row * S::TILE + j] * kLog2e);
      mc = fmaxf(mc, s[j]);
    }
    const float m_new = fmaxf(m, mc);
    if (m_new == -INFINITY) continue;  // nothing but padded keys so far (cannot happen for k0 < N)
    const float alpha = exp2f(m - m_new);
    l *= alpha;
#pragma unroll
    for (int e = 0; e < S::E; ++e) acc[e] *= alpha;
#pragma unroll
    for (int j = 0; j < kKC; ++j) {
      const float pj = exp2f(s[j] - m_new);
      l += pj;
      const float4* vr = reinterpret_cast<const float4*>(vs + j * S::ROW + part * S::SLICE);
#pragma unroll
      for (int e4 = 0; e4 < S::E / 4; ++e4) {
        const float4 vv = vr[e4];
        acc[4 * e4] = fmaf(pj, vv.x, acc[4 * e4]);
        acc[4 * e4 + 1] = fmaf(pj, vv.y, acc[4 * e4 + 1]);
        acc[4 * e4 + 2] = fmaf(pj, vv.z, acc[4 * e4 + 2]);
        acc[4 * e4 + 3] = fmaf(pj, vv.w, acc[4 * e4 + 3]);
      }
    }
    m = m_new;
  }
  if (bad_index) atomicOr(&g_device_error, 2);
  if (!valid) return;
  const float inv = 1.f / l;
  T* og = static_cast<T*>(p.out) + b * p.os_b + h * p.os_h + (long long)i * p.os_n + part * S::E;
#pragma unroll
  for (int e = 0; e < S::E; ++e) og[e] = from_f32<T>(acc[e] * inv);
}

template <typename T, int D>
int launch_simt(const SimtParams& p, long long blocks, cudaStream_t stream) {
  using S = Shape<D>;
  auto kern = window_attention_simt_kernel<T, D>;
  if (S::SMEM > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
    if (e != cudaSuccess) return set_cuda_error(e, "attention (simt) smem attribute");
  }
  kern<<<unsigned(blocks), kThreads, S::SMEM, stream>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "attention (simt) launch");
  return kOk;
}

template <typename T>
int dispatch_head_dim(const SimtParams& p, int head_dim, cudaStream_t stream) {
  const long long blocks = (long long)p.B * p.H * p.QB;
  switch (head_dim) {
    case 16: return launch_simt<T, 16>(p, blocks, stream);
    case 32: return launch_simt<T, 32>(p, blocks, stream);
    case 64: return launch_simt<T, 64>(p, blocks, stream);
    case 128: return launch_simt<T, 128>(p, blocks, stream);
    default: return launch_simt<T, 256>(p, blocks, stream);
  }
}

int rows_per_block(int head_dim) {
  switch (head_dim) {
    case 16: return Shape<16>::R;
    case 32: return Shape<32>::R;
    case 64: return Shape<64>::R;
    case 128: return Shape<128>::R;
    default: return Shape<256>::R;
  }
}

}  // namespace

bool simt_attention_head_dim(int64_t head_dim) {
  return head_dim == 16 || head_dim == 32 || head_dim == 64 || head_dim == 128 || head_dim == 256;
}

int launch_window_attention_simt(const AttnArgs& a, cudaStream_t stream) {
  if (!simt_attention_head_dim(a.head_dim))
    return set_error(kErrUnsupported,
                     "fused_swin_attention requires a power-of-two head_dim between 16 and 256");
  SimtParams p{};
  p.q = a.q;
  p.k = a.k;
  p.v = a.v;
  p.out = a.out;
  p.qs_b = a.qkv_stride_b;
  p.qs_h = a.qkv_stride_h;
  p.qs_n = a.qkv_stride_n;
  p.os_b = a.out_stride_b;
  p.os_h = a.out_stride_h;
  p.os_n = a.out_stride_n;
  p.bias = a.bias;
  p.table = a.table;
  p.index = reinterpret_cast<const long long*>(a.index);
  p.table_rows = a.table_rows;
  p.index_stride = a.index_stride;
  p.bias_from_table = a.bias_from_table ? 1 : 0;
  p.table_f32 = a.table_f32 ? 1 : 0;
  p.mask = a.mask;
  p.boundary = a.boundary;
  p.mask_windows = a.mask ? int(a.mask_windows) : 1;
  p.analytic = a.analytic ? 1 : 0;
  p.nwd = int(a.nwin[0]);
  p.nwh = int(a.nwin[1]);
  p.nww = int(a.nwin[2]);
  p.wsd = int(a.win[0]);
  p.wsh = int(a.win[1]);
  p.wsw = int(a.win[2]);
  p.ssd = int(a.shift[0]);
  p.ssh = int(a.shift[1]);
  p.ssw = int(a.shift[2]);
  if (!a.analytic) p.nwd = p.nwh = p.nww = p.wsd = p.wsh = p.wsw = 1;
  p.B = int(a.B);
  p.H = int(a.H);
  p.N = int(a.N);
  const int rows = rows_per_block(int(a.head_dim));
  p.QB = int((a.N + rows - 1) / rows);
  p.scale = a.scale;
  if ((long long)p.B * p.H * p.QB > 0x7fffffffLL)
    return set_error(kErrInvalid, "too many windows x heads for one launch");
  if (a.dtype == kF32) return dispatch_head_dim<float>(p, int(a.head_dim), stream);
  if (a.dtype == kBF16) return dispatch_head_dim<__nv_bfloat16>(p, int(a.head_dim), stream);
  return dispatch_head_dim<__half>(p, int(a.head_dim), stream);
}

}  // namespace crumpet
