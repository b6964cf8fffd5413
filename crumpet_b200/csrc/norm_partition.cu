// crumpet_b200: the memory passes around the window attention of a Swin block,
// fused.
//
// The reference's patched block (torch-ext/crumpet/monai_patch.py:79-111) runs
//   norm1 (LayerNorm; fp32 under fp16 autocast) -> F.pad of D/H/W up to a window
//   multiple -> roll + partition -> [qkv Linear casts to fp16] -> attention ->
//   unpartition + roll back -> crop of the padding -> residual add (MONAI block)
// as separate full-volume passes.  Two kernels replace them:
//
// norm_shift_partition: out[b*nW + win, loc, :] =
//     LN(x[b, s_d, s_h, s_w, :])  when s lies inside the D x H x W volume,
//     0                            when s lies in the padding (F.pad comes after
//                                  the norm, so padded tokens are exact zeros),
//   with s = (win_coord*ws + loc_coord + ss) mod padded_dim per axis -- the
//   geometry of partition.cu on the padded grid Dp = ceil(D/ws)*ws.
//   LN(v) = (v - mean) * rsqrt(var + eps) * weight + bias over C channels in fp32,
//   biased variance (torch.nn.LayerNorm), rounded once to the output type, which
//   may differ from the input type (fp16 out for the qkv Linear under autocast).
//
// unshift_unpartition_crop: out[b, d, h, w, :] (+ residual[b, d, h, w, :]) =
//     windows[b*nW + win(p), loc(p), :],  p = (d - ss) mod Dp, ... per axis,
//   for the unpadded volume only: padded tokens are never read, the cropped
//   volume is written directly.  The residual add happens in fp32 and is
//   rounded once, as torch's elementwise add for half types.
#include "common.cuh"
#include "kernels.h"

namespace crumpet {

namespace {

constexpr int kThreads = 128;  // 256 and 512 measured slower for the LayerNorm kernels
// LayerNorm kernel work split: a token's C channels are 8-channel groups spread
// over L lanes (L a power of two, the smallest with L * kGroupsPerLane >= C/8),
// kGroupsPerLane groups per lane, and each L-lane group normalises
// kTokensPerGroup tokens with all their loads in flight before any arithmetic.
constexpr int kGroupsPerLane = 3;
constexpr int kTokensPerGroup = 2;
constexpr int kMaxC = 32 * kGroupsPerLane * 8;  // L <= 32: C <= 768
// Patch merging normalises 8C channels; above 768 it runs 32 lanes per token
// with 6 or 12 groups per lane (8C <= 1536 / 3072) and one token per lane group.
constexpr int kMaxMergeC = 32 * 12 * 8;  // 8C <= 3072

struct BlockGeom {
  uint32_t D, H, W;        // unpadded volume
  uint32_t Dp, Hp, Wp;     // padded grid (window multiples)
  uint32_t wd, wh, ww, sd, sh, sw;
  uint32_t nwh, nww, nw, N, C, groups;  // groups = C / 8
  uint32_t tokens;         // output tokens of this launch (B_slice * nW * N, or B_slice * D*H*W)
  DivMod32 f_N, f_nw, f_nww, f_nwh, f_ww, f_wh, f_wd;
  DivMod32 f_W, f_H, f_D;  // unpadded volume
  float eps;
};

// 8 consecutive channels: raw 16/32-byte load, conversion to fp32, store.
template <typename T>
struct Io;
template <>
struct Io<float> {
  struct Raw {
    uint4 a, b;
  };
  static __device__ __forceinline__ Raw load(const float* p) {
    return Raw{ldg_stream(reinterpret_cast<const uint4*>(p)),
               ldg_stream(reinterpret_cast<const uint4*>(p) + 1)};
  }
  static __device__ __forceinline__ void to_float(const Raw& r, float (&v)[8]) {
    const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(w[i]);
  }
  static __device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
    stg(reinterpret_cast<uint4*>(p), make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]),
                                                __float_as_uint(v[2]), __float_as_uint(v[3])));
    stg(reinterpret_cast<uint4*>(p) + 1,
        make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]), __float_as_uint(v[6]),
                   __float_as_uint(v[7])));
  }
};
template <>
struct Io<__half> {
  struct Raw {
    uint4 a;
  };
  static __device__ __forceinline__ Raw load(const __half* p) {
    return Raw{ldg_stream(reinterpret_cast<const uint4*>(p))};
  }
  static __device__ __forceinline__ void to_float(const Raw& r, float (&v)[8]) {
    const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void store8(__half* p, const float (&v)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    stg(reinterpret_cast<uint4*>(p), make_uint4(w[0], w[1], w[2], w[3]));
  }
};
template <>
struct Io<__nv_bfloat16> {
  struct Raw {
    uint4 a;
  };
  static __device__ __forceinline__ Raw load(const __nv_bfloat16* p) {
    return Raw{ldg_stream(reinterpret_cast<const uint4*>(p))};
  }
  static __device__ __forceinline__ void to_float(const Raw& r, float (&v)[8]) {
    const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
  static __device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    stg(reinterpret_cast<uint4*>(p), make_uint4(w[0], w[1], w[2], w[3]));
  }
};

// Token t's source voxel: ((b*D + s_d)*H + s_h)*W + s_w, or "padding".
__device__ __forceinline__ bool token_source(const BlockGeom& g, uint32_t token, uint64_t& src) {
  uint32_t bw, loc, b, win, t, iw, id, ih, t2, lw, ld, lh;
  g.f_N.divmod(token, bw, loc);
  g.f_nw.divmod(bw, b, win);
  g.f_nww.divmod(win, t, iw);
  g.f_nwh.divmod(t, id, ih);
  g.f_ww.divmod(loc, t2, lw);
  g.f_wh.divmod(t2, ld, lh);
  uint32_t sd = id * g.wd + ld + g.sd;
  uint32_t sh = ih * g.wh + lh + g.sh;
  uint32_t sw = iw * g.ww + lw + g.sw;
  sd -= (sd >= g.Dp) ? g.Dp : 0u;
  sh -= (sh >= g.Hp) ? g.Hp : 0u;
  sw -= (sw >= g.Wp) ? g.Wp : 0u;
  src = ((uint64_t(b) * g.D + sd) * g.H + sh) * g.W + sw;
  return sd < g.D && sh < g.H && sw < g.W;
}

template <int L>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int off = L / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// (mean, rstd) of one token whose channels are spread over an L-lane group: this
// lane holds up to G 8-channel groups (bit k of `valid`: group k holds
// data; the others count as zeros).  Sums in packed fp32 pairs, then the lane
// group's shuffles; biased variance, as torch.nn.LayerNorm.
template <int L, int G>
__device__ __forceinline__ float2 token_stats(const float (&v)[G][8], uint32_t valid, float inv_c,
                                              float eps) {
  float2 s = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < G; ++k)
    if ((valid >> k) & 1u)
#pragma unroll
      for (int e = 0; e < 8; e += 2) s = __fadd2_rn(s, make_float2(v[k][e], v[k][e + 1]));
  const float mean = group_sum<L>(s.x + s.y) * inv_c;
  const float2 nm = make_float2(-mean, -mean);
  float2 q = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < G; ++k)
    if ((valid >> k) & 1u)
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float2 d = __fadd2_rn(make_float2(v[k][e], v[k][e + 1]), nm);
        q = __ffma2_rn(d, d, q);
      }
  return make_float2(mean, rsqrtf(group_sum<L>(q.x + q.y) * inv_c + eps));
}

// gamma and beta of one 8-channel group, loaded once and applied to several tokens:
// y = (v - mean) * rstd * gamma + beta in packed pairs (each lane of a pair rounds
// exactly as the scalar expression would).
struct Affine8 {
  float2 gm[4], bt[4];
  static __device__ __forceinline__ Affine8 load(const float* __restrict__ gamma8,
                                                 const float* __restrict__ beta8) {
    const float4 ga = __ldg(reinterpret_cast<const float4*>(gamma8));
    const float4 gb = __ldg(reinterpret_cast<const float4*>(gamma8) + 1);
    const float4 ba = __ldg(reinterpret_cast<const float4*>(beta8));
    const float4 bb = __ldg(reinterpret_cast<const float4*>(beta8) + 1);
    return Affine8{{make_float2(ga.x, ga.y), make_float2(ga.z, ga.w), make_float2(gb.x, gb.y),
                    make_float2(gb.z, gb.w)},
                   {make_float2(ba.x, ba.y), make_float2(ba.z, ba.w), make_float2(bb.x, bb.y),
                    make_float2(bb.z, bb.w)}};
  }
  // the same from a shared-memory copy of gamma / beta
  static __device__ __forceinline__ Affine8 load_shared(const float* gamma8, const float* beta8) {
    const float4 ga = reinterpret_cast<const float4*>(gamma8)[0];
    const float4 gb = reinterpret_cast<const float4*>(gamma8)[1];
    const float4 ba = reinterpret_cast<const float4*>(beta8)[0];
    const float4 bb = reinterpret_cast<const float4*>(beta8)[1];
    return Affine8{{make_float2(ga.x, ga.y), make_float2(ga.z, ga.w), make_float2(gb.x, gb.y),
                    make_float2(gb.z, gb.w)},
                   {make_float2(ba.x, ba.y), make_float2(ba.z, ba.w), make_float2(bb.x, bb.y),
                    make_float2(bb.z, bb.w)}};
  }
  __device__ __forceinline__ void apply(const float (&v)[8], float2 st, float (&y)[8]) const {
    const float2 nm = make_float2(-st.x, -st.x), rs = make_float2(st.y, st.y);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __fmul2_rn(__fadd2_rn(make_float2(v[2 * i], v[2 * i + 1]), nm), rs);
      const float2 r = __ffma2_rn(t, gm[i], bt[i]);
      y[2 * i] = r.x;
      y[2 * i + 1] = r.y;
    }
  }
};

// gamma and beta of `n` channels copied into shared memory (gb[0..n) and gb[cap..cap+n)) by
// the whole block: the normalise step then reads them with short-latency shared loads
// instead of L1 hits on its critical path (norm + partition 32.8 -> 30.3 us, crop + norm2
// 53.2 -> 52.2 us at stage 1; patch merging, whose blocks cover only 32 tokens of 8C
// channels, is faster without it).  All threads of the block must call this.
__device__ __forceinline__ void stage_affine(float* gb, uint32_t cap,
                                             const float* __restrict__ gamma,
                                             const float* __restrict__ beta, uint32_t n) {
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    gb[i] = __ldg(gamma + i);
    gb[cap + i] = __ldg(beta + i);
  }
  __syncthreads();
}

// The index math of a lane group's NT tokens (first + j * stride) is
// done once per token -- by lane j of the group for token j -- and broadcast to the
// group's other lanes, instead of by every lane.  `fn(token, payload)` returns
// whether the token has a source and sets its 64-bit payload.  All 32 lanes of
// the warp must call this.
template <int L, int NT, typename SourceFn>
__device__ __forceinline__ void group_sources(uint32_t first, uint32_t stride, SourceFn fn,
                                              uint64_t (&payload)[NT], bool (&ok)[NT]) {
  if constexpr (L >= NT) {
    const uint32_t lane = threadIdx.x & 31u, sub = lane % L;
    uint64_t mine = 0;
    int mine_ok = 0;
    if (sub < uint32_t(NT)) mine_ok = fn(first + sub * stride, mine) ? 1 : 0;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      payload[j] = __shfl_sync(0xffffffffu, mine, int(lane - sub) + j);
      ok[j] = __shfl_sync(0xffffffffu, mine_ok, int(lane - sub) + j) != 0;
    }
  } else {
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      payload[j] = 0;
      ok[j] = fn(first + j * stride, payload[j]);
    }
  }
}

// Lane `sub` of an L-lane group owns channel groups sub, sub + L, sub + 2L of
// its tokens; the group's tokens in one block step are consecutive output
// tokens, so a warp reads and writes contiguous rows.
template <typename TIn, typename TOut, int L>
__global__ void __launch_bounds__(kThreads)
norm_shift_partition_kernel(TOut* __restrict__ out, const TIn* __restrict__ x,
                            const float* __restrict__ gamma, const float* __restrict__ beta,
                            const BlockGeom g) {
  constexpr uint32_t kGroups = kThreads / L;  // lane groups per block
  const uint32_t sub = threadIdx.x % L;
  __shared__ __align__(16) float gb_s[2 * kMaxC];
  stage_affine(gb_s, kMaxC, gamma, beta, g.C);
  const uint32_t first = blockIdx.x * (kGroups * kTokensPerGroup) + threadIdx.x / L;
  uint64_t src[kTokensPerGroup];
  bool inside[kTokensPerGroup];
  group_sources<L>(first, kGroups,
                   [&](uint32_t t, uint64_t& s) { return t < g.tokens && token_source(g, t, s); },
                   src, inside);
  typename Io<TIn>::Raw raw[kTokensPerGroup][kGroupsPerLane];
#pragma unroll
  for (int j = 0; j < kTokensPerGroup; ++j) {
#pragma unroll
    for (int k = 0; k < kGroupsPerLane; ++k) {
      const uint32_t grp = sub + k * L;
      if (inside[j] && grp < g.groups) raw[j][k] = Io<TIn>::load(x + src[j] * g.C + grp * 8);
    }
  }
  const float inv_c = 1.f / float(g.C);
  // one token at a time: keeping a second token's fp32 values live for a shared gamma /
  // beta load costs registers (80 instead of 64) and resident blocks, and is slower here
#pragma unroll
  for (int j = 0; j < kTokensPerGroup; ++j) {
    const uint32_t token = first + j * kGroups;
    float v[kGroupsPerLane][8];
    uint32_t valid = 0;
#pragma unroll
    for (int k = 0; k < kGroupsPerLane; ++k) {
      if (inside[j] && sub + k * L < g.groups) {
        Io<TIn>::to_float(raw[j][k], v[k]);
        valid |= 1u << k;
      }
    }
    // every lane takes part in the shuffles (padding and dead tokens add zeros)
    const float2 st = token_stats<L>(v, valid, inv_c, g.eps);
    if (token >= g.tokens) continue;
    TOut* dst = out + uint64_t(token) * g.C;
#pragma unroll
    for (int k = 0; k < kGroupsPerLane; ++k) {
      const uint32_t grp = sub + k * L;
      if (grp >= g.groups) continue;
      float y[8];
      if (inside[j]) {
        Affine8::load_shared(gb_s + grp * 8, gb_s + kMaxC + grp * 8).apply(v[k], st, y);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = 0.f;  // F.pad after the norm: zeros
      }
      Io<TOut>::store8(dst + grp * 8, y);
    }
  }
}

// a + b per 32-bit word, in fp32, rounded once (torch's add for half types).
template <typename T>
__device__ __forceinline__ uint32_t add_word(uint32_t a, uint32_t b);
template <>
__device__ __forceinline__ uint32_t add_word<float>(uint32_t a, uint32_t b) {
  return __float_as_uint(__uint_as_float(a) + __uint_as_float(b));
}
template <>
__device__ __forceinline__ uint32_t add_word<__half>(uint32_t a, uint32_t b) {
  const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&a));
  const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&b));
  const __half2 r = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
  return *reinterpret_cast<const uint32_t*>(&r);
}
template <>
__device__ __forceinline__ uint32_t add_word<__nv_bfloat16>(uint32_t a, uint32_t b) {
  const float lo = __uint_as_float(a << 16) + __uint_as_float(b << 16);
  const float hi = __uint_as_float(a & 0xFFFF0000u) + __uint_as_float(b & 0xFFFF0000u);
  const __nv_bfloat162 r = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&r);
}

template <typename T, int VB>
__device__ __forceinline__ typename VecT<VB>::type add_vec(typename VecT<VB>::type a,
                                                          typename VecT<VB>::type b) {
  if constexpr (VB == 16) {
    return make_uint4(add_word<T>(a.x, b.x), add_word<T>(a.y, b.y), add_word<T>(a.z, b.z),
                      add_word<T>(a.w, b.w));
  } else if constexpr (VB == 8) {
    return make_uint2(add_word<T>(a.x, b.x), add_word<T>(a.y, b.y));
  } else {
    return add_word<T>(a, b);
  }
}

// One thread per output vector of the cropped volume.
template <typename T, int VB, bool RES>
__global__ void __launch_bounds__(kThreads)
unshift_unpartition_crop_kernel(typename VecT<VB>::type* __restrict__ out,
                                const typename VecT<VB>::type* __restrict__ windows,
                                const typename VecT<VB>::type* __restrict__ residual,
                                const BlockGeom g, uint32_t cv, DivMod32 f_cv, DivMod32 f_W,
                                DivMod32 f_H, DivMod32 f_D, uint32_t total) {
  const uint32_t o = blockIdx.x * kThreads + threadIdx.x;
  if (o >= total) return;
  uint32_t p, v, t, w, t2, h, b, d, id, ld, ih, lh, iw, lw;
  f_cv.divmod(o, p, v);
  f_W.divmod(p, t, w);
  f_H.divmod(t, t2, h);
  f_D.divmod(t2, b, d);
  d = (d >= g.sd) ? d - g.sd : d + g.Dp - g.sd;
  h = (h >= g.sh) ? h - g.sh : h + g.Hp - g.sh;
  w = (w >= g.sw) ? w - g.sw : w + g.Wp - g.sw;
  g.f_wd.divmod(d, id, ld);
  g.f_wh.divmod(h, ih, lh);
  g.f_ww.divmod(w, iw, lw);
  const uint32_t win = (id * g.nwh + ih) * g.nww + iw;
  const uint32_t loc = (ld * g.wh + lh) * g.ww + lw;
  const uint64_t src = (uint64_t(b) * g.nw + win) * g.N * cv + uint64_t(loc) * cv + v;
  auto val = ldg_stream(windows + src);
  if constexpr (RES) val = add_vec<T, VB>(ldg_stream(residual + o), val);
  stg(out + o, val);
}

// Rounds an fp32 value to T and back (the value a T tensor would hold).
template <typename T>
__device__ __forceinline__ float round_to(float v);
template <>
__device__ __forceinline__ float round_to<float>(float v) { return v; }
template <>
__device__ __forceinline__ float round_to<__half>(float v) {
  return __half2float(__float2half_rn(v));
}
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// Unpartition + roll back + crop + residual, and the LayerNorm of the result (the
// MLP half's norm2) in the same pass.  One output token (b, d, h, w) of the cropped
// volume per L-lane group, kTokensPerGroup tokens per group with all loads in
// flight first.  out = T(residual + window row), normed = LN(out) in TN, where the
// norm reads the rounded T values, as a separate norm over the stored tensor would.
template <typename T, typename TN, int L>
__global__ void __launch_bounds__(kThreads)
unshift_crop_norm_kernel(T* __restrict__ out, TN* __restrict__ normed,
                         const T* __restrict__ windows, const T* __restrict__ residual,
                         const float* __restrict__ gamma, const float* __restrict__ beta,
                         const BlockGeom g) {
  constexpr uint32_t kGroups = kThreads / L;
  const uint32_t sub = threadIdx.x % L;
  __shared__ __align__(16) float gb_s[2 * kMaxC];
  stage_affine(gb_s, kMaxC, gamma, beta, g.C);
  const uint32_t first = blockIdx.x * (kGroups * kTokensPerGroup) + threadIdx.x / L;
  uint64_t src[kTokensPerGroup];
  bool live[kTokensPerGroup];
  group_sources<L>(
      first, kGroups,
      [&](uint32_t token, uint64_t& s) {
        if (token >= g.tokens) return false;
        uint32_t t, w, t2, h, b, d, id, ld, ih, lh, iw, lw;
        g.f_W.divmod(token, t, w);
        g.f_H.divmod(t, t2, h);
        g.f_D.divmod(t2, b, d);
        d = (d >= g.sd) ? d - g.sd : d + g.Dp - g.sd;
        h = (h >= g.sh) ? h - g.sh : h + g.Hp - g.sh;
        w = (w >= g.sw) ? w - g.sw : w + g.Wp - g.sw;
        g.f_wd.divmod(d, id, ld);
        g.f_wh.divmod(h, ih, lh);
        g.f_ww.divmod(w, iw, lw);
        const uint32_t win = (id * g.nwh + ih) * g.nww + iw;
        const uint32_t loc = (ld * g.wh + lh) * g.ww + lw;
        s = (uint64_t(b) * g.nw + win) * g.N + loc;
        return true;
      },
      src, live);
  typename Io<T>::Raw rw[kTokensPerGroup][kGroupsPerLane], rr[kTokensPerGroup][kGroupsPerLane];
#pragma unroll
  for (int j = 0; j < kTokensPerGroup; ++j) {
    const uint32_t token = first + j * kGroups;
#pragma unroll
    for (int k = 0; k < kGroupsPerLane; ++k) {
      const uint32_t grp = sub + k * L;
      if (live[j] && grp < g.groups) {
        rw[j][k] = Io<T>::load(windows + src[j] * g.C + grp * 8);
        if (residual) rr[j][k] = Io<T>::load(residual + uint64_t(token) * g.C + grp * 8);
      }
    }
  }
  const float inv_c = 1.f / float(g.C);
  float v[kTokensPerGroup][kGroupsPerLane][8];
  float2 st[kTokensPerGroup];
#pragma unroll
  for (int j = 0; j < kTokensPerGroup; ++j) {
    const uint32_t token = first + j * kGroups;
    uint32_t valid = 0;
#pragma unroll
    for (int k = 0; k < kGroupsPerLane; ++k) {
      const uint32_t grp = sub + k * L;
      if (live[j] && grp < g.groups) {
        Io<T>::to_float(rw[j][k], v[j][k]);
        if (residual) {
          float r[8];
          Io<T>::to_float(rr[j][k], r);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[j][k][e] = round_to<T>(r[e] + v[j][k][e]);
        }
        Io<T>::store8(out + uint64_t(token) * g.C + grp * 8, v[j][k]);
        valid |= 1u << k;
      }
    }
    st[j] = token_stats<L>(v[j], valid, inv_c, g.eps);
  }
#pragma unroll
  for (int k = 0; k < kGroupsPerLane; ++k) {
    const uint32_t grp = sub + k * L;
    if (grp >= g.groups) continue;
    const Affine8 ab = Affine8::load_shared(gb_s + grp * 8, gb_s + kMaxC + grp * 8);
#pragma unroll
    for (int j = 0; j < kTokensPerGroup; ++j) {
      if (!live[j]) continue;
      float y[8];
      ab.apply(v[j][k], st[j], y);
      Io<TN>::store8(normed + uint64_t(first + j * kGroups) * g.C + grp * 8, y);
    }
  }
}

// Patch merging: out[b, d2, h2, w2, :] = LN(cat_p x[b, 2 d2 + i_p, 2 h2 + j_p, 2 w2 + k_p, :])
// over the 8C concatenated channels (part order from `parts`, zero rows past odd
// dims, as the module's F.pad).  One output voxel per L-lane group.
struct MergeGeom {
  uint32_t D, H, W, C, D2, H2, W2, groups, part_groups;  // groups = 8C/8, part_groups = C/8
  uint32_t tokens;
  DivMod32 f_W2, f_H2, f_D2, f_pg;
  uint32_t parts;  // 3 bits (i | j << 1 | k << 2) per part, part p at bits 3p..3p+2
  float eps;
};

// G groups of 8 channels per lane, NT tokens per L-lane group.
template <typename TIn, typename TOut, int L, int G, int NT>
__global__ void __launch_bounds__(kThreads)
patch_merge_norm_kernel(TOut* __restrict__ out, const TIn* __restrict__ x,
                        const float* __restrict__ gamma, const float* __restrict__ beta,
                        const MergeGeom g) {
  constexpr uint32_t kGroups = kThreads / L;
  const uint32_t sub = threadIdx.x % L;
  const uint32_t first = blockIdx.x * (kGroups * NT) + threadIdx.x / L;
  // per output voxel: the input voxel index of its (0, 0, 0) neighbour, with bits
  // 61..63 set when the +1 neighbour along D / H / W lies inside the volume
  uint64_t base[NT];
  bool live[NT];
  group_sources<L>(
      first, kGroups,
      [&](uint32_t token, uint64_t& s) {
        if (token >= g.tokens) return false;
        uint32_t t, w2, t2, h2, b, d2;
        g.f_W2.divmod(token, t, w2);
        g.f_H2.divmod(t, t2, h2);
        g.f_D2.divmod(t2, b, d2);
        const uint64_t edges = uint64_t(2 * d2 + 1 < g.D) | (uint64_t(2 * h2 + 1 < g.H) << 1) |
                               (uint64_t(2 * w2 + 1 < g.W) << 2);
        s = (((uint64_t(b) * g.D + 2 * d2) * g.H + 2 * h2) * g.W + 2 * w2) | (edges << 61);
        return true;
      },
      base, live);
  uint32_t inb[NT];  // bit k: channel group sub + k*L lies inside the volume
  typename Io<TIn>::Raw raw[NT][G];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    inb[j] = 0;
    const uint32_t edges = uint32_t(base[j] >> 61);
    const uint64_t v0 = base[j] & ((uint64_t(1) << 61) - 1);
#pragma unroll
    for (int k = 0; k < G; ++k) {
      const uint32_t grp = sub + k * L;
      if (live[j] && grp < g.groups) {
        uint32_t part, cg;
        g.f_pg.divmod(grp, part, cg);
        const uint32_t code = (g.parts >> (3 * part)) & 7u;
        if ((code & ~edges) == 0) {  // every +1 offset of this part stays inside the volume
          const uint64_t v = v0 + ((code & 1u) * g.H + ((code >> 1) & 1u)) * g.W + (code >> 2);
          raw[j][k] = Io<TIn>::load(x + v * g.C + cg * 8);
          inb[j] |= 1u << k;
        }
      }
    }
  }
  const float inv_c = 1.f / float(8 * g.C);
  float v[NT][G][8];
  float2 st[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    uint32_t valid = 0;
#pragma unroll
    for (int k = 0; k < G; ++k) {
      if ((inb[j] >> k) & 1u) {
        Io<TIn>::to_float(raw[j][k], v[j][k]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[j][k][e] = 0.f;  // padding rows (and unused groups)
      }
      if (sub + k * L < g.groups) valid |= 1u << k;
    }
    st[j] = token_stats<L>(v[j], valid, inv_c, g.eps);
  }
#pragma unroll
  for (int k = 0; k < G; ++k) {
    const uint32_t grp = sub + k * L;
    if (grp >= g.groups) continue;
    const Affine8 ab = Affine8::load(gamma + grp * 8, beta + grp * 8);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      if (!live[j]) continue;
      float y[8];
      ab.apply(v[j][k], st[j], y);
      Io<TOut>::store8(out + uint64_t(first + j * kGroups) * (8 * g.C) + grp * 8, y);
    }
  }
}

int check_geometry(int64_t B, int64_t D, int64_t H, int64_t W, int64_t C, const int64_t* ws,
                   const int64_t* ss) {
  const int64_t dims[3] = {D, H, W};
  if (B < 0 || C < 0) return set_error(kErrInvalid, "B and C must be non-negative");
  for (int a = 0; a < 3; ++a) {
    if (dims[a] <= 0) return set_error(kErrInvalid, "D, H and W must be positive");
    if (ws[a] <= 0) return set_error(kErrInvalid, "window_size values must be positive");
    if (ss[a] < 0 || ss[a] >= ws[a])
      return set_error(kErrInvalid, "shift_size must satisfy 0 <= shift < window_size");
  }
  int64_t padded = 1;
  for (int a = 0; a < 3; ++a) padded *= (dims[a] + ws[a] - 1) / ws[a] * ws[a];
  if (padded >= (int64_t(1) << 31))
    return set_error(kErrInvalid, "padded D*H*W must be below 2^31");
  return kOk;
}

BlockGeom make_geom(int64_t D, int64_t H, int64_t W, int64_t C, const int64_t* ws,
                    const int64_t* ss) {
  BlockGeom g{};
  g.D = uint32_t(D);
  g.H = uint32_t(H);
  g.W = uint32_t(W);
  g.wd = uint32_t(ws[0]);
  g.wh = uint32_t(ws[1]);
  g.ww = uint32_t(ws[2]);
  g.Dp = (g.D + g.wd - 1) / g.wd * g.wd;
  g.Hp = (g.H + g.wh - 1) / g.wh * g.wh;
  g.Wp = (g.W + g.ww - 1) / g.ww * g.ww;
  g.sd = uint32_t(ss[0]);
  g.sh = uint32_t(ss[1]);
  g.sw = uint32_t(ss[2]);
  g.nwh = g.Hp / g.wh;
  g.nww = g.Wp / g.ww;
  g.nw = (g.Dp / g.wd) * g.nwh * g.nww;
  g.N = g.wd * g.wh * g.ww;
  g.C = uint32_t(C);
  g.groups = g.C / 8;
  g.f_N = DivMod32::make(g.N);
  g.f_nw = DivMod32::make(g.nw);
  g.f_nww = DivMod32::make(g.nww);
  g.f_nwh = DivMod32::make(g.nwh);
  g.f_ww = DivMod32::make(g.ww);
  g.f_wh = DivMod32::make(g.wh);
  g.f_wd = DivMod32::make(g.wd);
  g.f_W = DivMod32::make(g.W);
  g.f_H = DivMod32::make(g.H);
  g.f_D = DivMod32::make(g.D);
  return g;
}

template <typename TIn, typename TOut>
cudaError_t launch_norm(void* out, const void* x, const float* gamma, const float* beta,
                        const BlockGeom& g, cudaStream_t stream) {
  int lanes = 1;
  while (uint32_t(lanes * kGroupsPerLane) < g.groups) lanes *= 2;
  const uint32_t per_block = uint32_t(kThreads / lanes) * kTokensPerGroup;
  const uint32_t blocks = (g.tokens + per_block - 1) / per_block;
  auto o = static_cast<TOut*>(out);
  auto xi = static_cast<const TIn*>(x);
  switch (lanes) {
    case 1: norm_shift_partition_kernel<TIn, TOut, 1><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
    case 2: norm_shift_partition_kernel<TIn, TOut, 2><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
    case 4: norm_shift_partition_kernel<TIn, TOut, 4><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
    case 8: norm_shift_partition_kernel<TIn, TOut, 8><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
    case 16: norm_shift_partition_kernel<TIn, TOut, 16><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
    default: norm_shift_partition_kernel<TIn, TOut, 32><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
  }
  return cudaGetLastError();
}

template <typename TIn>
cudaError_t launch_norm_out(int out_dtype, void* out, const void* x, const float* gamma,
                            const float* beta, const BlockGeom& g, cudaStream_t stream) {
  if (out_dtype == kF32) return launch_norm<TIn, float>(out, x, gamma, beta, g, stream);
  if (out_dtype == kF16) return launch_norm<TIn, __half>(out, x, gamma, beta, g, stream);
  return launch_norm<TIn, __nv_bfloat16>(out, x, gamma, beta, g, stream);
}

template <typename T, int VB, bool RES>
cudaError_t launch_crop_t(void* out, const void* windows, const void* residual, const BlockGeom& g,
                          uint32_t cv, uint32_t batches, cudaStream_t stream) {
  using V = typename VecT<VB>::type;
  const uint32_t total = batches * g.D * g.H * g.W * cv;
  const uint32_t blocks = (total + kThreads - 1) / kThreads;
  unshift_unpartition_crop_kernel<T, VB, RES><<<blocks, kThreads, 0, stream>>>(
      static_cast<V*>(out), static_cast<const V*>(windows), static_cast<const V*>(residual), g, cv,
      DivMod32::make(cv), DivMod32::make(g.W), DivMod32::make(g.H), DivMod32::make(g.D), total);
  return cudaGetLastError();
}

template <typename T, bool RES>
cudaError_t launch_crop_vb(int vb, void* out, const void* windows, const void* residual,
                           const BlockGeom& g, uint32_t cv, uint32_t batches,
                           cudaStream_t stream) {
  switch (vb) {
    case 16: return launch_crop_t<T, 16, RES>(out, windows, residual, g, cv, batches, stream);
    case 8: return launch_crop_t<T, 8, RES>(out, windows, residual, g, cv, batches, stream);
    default: return launch_crop_t<T, 4, RES>(out, windows, residual, g, cv, batches, stream);
  }
}

}  // namespace

int launch_norm_shift_partition(void* out, int out_dtype, const void* x, int in_dtype,
                                const float* gamma, const float* beta, float eps, int64_t B,
                                int64_t D, int64_t H, int64_t W, int64_t C, const int64_t* ws,
                                const int64_t* ss, cudaStream_t stream) {
  if (int e = check_geometry(B, D, H, W, C, ws, ss)) return e;
  if (C == 0 || C % 8 != 0 || C > kMaxC)
    return set_error(kErrUnsupported,
                     "norm_shift_partition_3d needs C a multiple of 8 and at most 768");
  if (ws[0] * ws[1] * ws[2] > 4096) return set_error(kErrInvalid, "window volume above 4096");
  if (B == 0) return kOk;
  if (!out || !x || !gamma || !beta) return set_error(kErrInvalid, "null tensor pointer");
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(x) |
       reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15u)
    return set_error(kErrInvalid, "tensors must be 16-byte aligned");
  BlockGeom g = make_geom(D, H, W, C, ws, ss);
  g.eps = eps;
  // batch slices keep every in-launch token index below 2^31
  const uint64_t per_batch = uint64_t(g.nw) * g.N;
  const uint64_t bmax = ((uint64_t(1) << 31) - 1) / per_batch;
  const int64_t in_row = C * dtype_size(in_dtype), out_row = C * dtype_size(out_dtype);
  for (int64_t b0 = 0; b0 < B; b0 += int64_t(bmax)) {
    const uint64_t nb = uint64_t(B - b0) < bmax ? uint64_t(B - b0) : bmax;
    g.tokens = uint32_t(nb * per_batch);
    const void* xs = static_cast<const uint8_t*>(x) + uint64_t(b0) * D * H * W * in_row;
    void* os = static_cast<uint8_t*>(out) + uint64_t(b0) * per_batch * out_row;
    cudaError_t err;
    if (in_dtype == kF32)
      err = launch_norm_out<float>(out_dtype, os, xs, gamma, beta, g, stream);
    else if (in_dtype == kF16)
      err = launch_norm_out<__half>(out_dtype, os, xs, gamma, beta, g, stream);
    else
      err = launch_norm_out<__nv_bfloat16>(out_dtype, os, xs, gamma, beta, g, stream);
    if (err != cudaSuccess) return set_cuda_error(err, "norm_shift_partition launch");
  }
  return kOk;
}

int launch_unshift_unpartition_crop(void* out, const void* windows, const void* residual,
                                    int dtype, int64_t B, int64_t D, int64_t H, int64_t W,
                                    int64_t C, const int64_t* ws, const int64_t* ss,
                                    cudaStream_t stream) {
  if (int e = check_geometry(B, D, H, W, C, ws, ss)) return e;
  if (B == 0 || C == 0) return kOk;
  if (!out || !windows) return set_error(kErrInvalid, "null tensor pointer");
  const int64_t row = C * dtype_size(dtype);
  const uintptr_t mis = reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(windows) |
                        reinterpret_cast<uintptr_t>(residual);
  int vb = 0;
  for (int c = 16; c >= 4; c /= 2) {
    if (row % c == 0 && mis % c == 0) {
      vb = c;
      break;
    }
  }
  if (vb == 0)
    return set_error(kErrUnsupported,
                     "unshift_unpartition_crop_3d needs 4-byte aligned rows and pointers");
  const BlockGeom g = make_geom(D, H, W, C, ws, ss);
  const uint32_t cv = uint32_t(row / vb);
  const uint64_t per_batch_vec = uint64_t(D) * H * W * cv;
  if (uint64_t(g.nw) * g.N * cv >= (uint64_t(1) << 32))
    return set_error(kErrInvalid, "one batch entry of windows is too large");
  const uint64_t bmax = ((uint64_t(1) << 31) - 1) / per_batch_vec;
  if (bmax == 0) return set_error(kErrInvalid, "one batch entry is too large for one launch");
  for (int64_t b0 = 0; b0 < B; b0 += int64_t(bmax)) {
    const uint64_t nb = uint64_t(B - b0) < bmax ? uint64_t(B - b0) : bmax;
    void* os = static_cast<uint8_t*>(out) + uint64_t(b0) * per_batch_vec * vb;
    const void* wsrc =
        static_cast<const uint8_t*>(windows) + uint64_t(b0) * g.nw * g.N * uint64_t(row);
    const void* rs =
        residual ? static_cast<const uint8_t*>(residual) + uint64_t(b0) * per_batch_vec * vb
                 : nullptr;
    cudaError_t err;
    if (residual == nullptr) {
      err = launch_crop_vb<float, false>(vb, os, wsrc, nullptr, g, cv, uint32_t(nb), stream);
    } else if (dtype == kF32) {
      err = launch_crop_vb<float, true>(vb, os, wsrc, rs, g, cv, uint32_t(nb), stream);
    } else if (dtype == kF16) {
      err = launch_crop_vb<__half, true>(vb, os, wsrc, rs, g, cv, uint32_t(nb), stream);
    } else {
      err = launch_crop_vb<__nv_bfloat16, true>(vb, os, wsrc, rs, g, cv, uint32_t(nb), stream);
    }
    if (err != cudaSuccess) return set_cuda_error(err, "unshift_unpartition_crop launch");
  }
  return kOk;
}


namespace {

template <typename T, typename TN>
cudaError_t launch_crop_norm_t(void* out, void* normed, const void* windows, const void* residual,
                               const float* gamma, const float* beta, const BlockGeom& g,
                               cudaStream_t stream) {
  int lanes = 1;
  while (uint32_t(lanes * kGroupsPerLane) < g.groups) lanes *= 2;
  const uint32_t per_block = uint32_t(kThreads / lanes) * kTokensPerGroup;
  const uint32_t blocks = (g.tokens + per_block - 1) / per_block;
  auto o = static_cast<T*>(out);
  auto n = static_cast<TN*>(normed);
  auto wi = static_cast<const T*>(windows);
  auto re = static_cast<const T*>(residual);
  switch (lanes) {
    case 1: unshift_crop_norm_kernel<T, TN, 1><<<blocks, kThreads, 0, stream>>>(o, n, wi, re, gamma, beta, g); break;
    case 2: unshift_crop_norm_kernel<T, TN, 2><<<blocks, kThreads, 0, stream>>>(o, n, wi, re, gamma, beta, g); break;
    case 4: unshift_crop_norm_kernel<T, TN, 4><<<blocks, kThreads, 0, stream>>>(o, n, wi, re, gamma, beta, g); break;
    case 8: unshift_crop_norm_kernel<T, TN, 8><<<blocks, kThreads, 0, stream>>>(o, n, wi, re, gamma, beta, g); break;
    case 16: unshift_crop_norm_kernel<T, TN, 16><<<blocks, kThreads, 0, stream>>>(o, n, wi, re, gamma, beta, g); break;
    default: unshift_crop_norm_kernel<T, TN, 32><<<blocks, kThreads, 0, stream>>>(o, n, wi, re, gamma, beta, g); break;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_crop_norm_n(int norm_dtype, void* out, void* normed, const void* windows,
                               const void* residual, const float* gamma, const float* beta,
                               const BlockGeom& g, cudaStream_t stream) {
  if (norm_dtype == kF32)
    return launch_crop_norm_t<T, float>(out, normed, windows, residual, gamma, beta, g, stream);
  if (norm_dtype == kF16)
    return launch_crop_norm_t<T, __half>(out, normed, windows, residual, gamma, beta, g, stream);
  return launch_crop_norm_t<T, __nv_bfloat16>(out, normed, windows, residual, gamma, beta, g,
                                               stream);
}

}  // namespace

int launch_unshift_unpartition_crop_norm(void* out, void* normed, int norm_dtype,
                                         const void* windows, const void* residual, int dtype,
                                         const float* gamma, const float* beta, float eps,
                                         int64_t B, int64_t D, int64_t H, int64_t W, int64_t C,
                                         const int64_t* ws, const int64_t* ss,
                                         cudaStream_t stream) {
  if (int e = check_geometry(B, D, H, W, C, ws, ss)) return e;
  if (C == 0 || C % 8 != 0 || C > kMaxC)
    return set_error(kErrUnsupported,
                     "unshift_unpartition_crop_norm_3d needs C a multiple of 8 and at most 768");
  if (B == 0) return kOk;
  if (!out || !normed || !windows || !gamma || !beta)
    return set_error(kErrInvalid, "null tensor pointer");
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(normed) |
       reinterpret_cast<uintptr_t>(windows) | reinterpret_cast<uintptr_t>(residual) |
       reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15u)
    return set_error(kErrInvalid, "tensors must be 16-byte aligned");
  BlockGeom g = make_geom(D, H, W, C, ws, ss);
  g.eps = eps;
  const uint64_t per_batch = uint64_t(D) * H * W;
  const uint64_t bmax = ((uint64_t(1) << 31) - 1) / per_batch;
  if (bmax == 0) return set_error(kErrInvalid, "one batch entry is too large for one launch");
  const int64_t row = C * dtype_size(dtype), nrow = C * dtype_size(norm_dtype);
  for (int64_t b0 = 0; b0 < B; b0 += int64_t(bmax)) {
    const uint64_t nb = uint64_t(B - b0) < bmax ? uint64_t(B - b0) : bmax;
    g.tokens = uint32_t(nb * per_batch);
    void* os = static_cast<uint8_t*>(out) + uint64_t(b0) * per_batch * row;
    void* ns = static_cast<uint8_t*>(normed) + uint64_t(b0) * per_batch * nrow;
    const void* wsrc =
        static_cast<const uint8_t*>(windows) + uint64_t(b0) * g.nw * g.N * uint64_t(row);
    const void* rs =
        residual ? static_cast<const uint8_t*>(residual) + uint64_t(b0) * per_batch * row : nullptr;
    cudaError_t err;
    if (dtype == kF32)
      err = launch_crop_norm_n<float>(norm_dtype, os, ns, wsrc, rs, gamma, beta, g, stream);
    else if (dtype == kF16)
      err = launch_crop_norm_n<__half>(norm_dtype, os, ns, wsrc, rs, gamma, beta, g, stream);
    else
      err = launch_crop_norm_n<__nv_bfloat16>(norm_dtype, os, ns, wsrc, rs, gamma, beta, g, stream);
    if (err != cudaSuccess) return set_cuda_error(err, "unshift_unpartition_crop_norm launch");
  }
  return kOk;
}


namespace {

template <typename TIn, typename TOut>
cudaError_t launch_merge_t(void* out, const void* x, const float* gamma, const float* beta,
                           const MergeGeom& g, cudaStream_t stream) {
  if (g.groups > uint32_t(32 * kGroupsPerLane)) {  // 8C > 768: 32 lanes, one token per group
    const uint32_t per_block = kThreads / 32;
    const uint32_t blocks = (g.tokens + per_block - 1) / per_block;
    auto o = static_cast<TOut*>(out);
    auto xi = static_cast<const TIn*>(x);
    if (g.groups <= 32 * 6)
      patch_merge_norm_kernel<TIn, TOut, 32, 6, 1><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g);
    else
      patch_merge_norm_kernel<TIn, TOut, 32, 12, 1><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g);
    return cudaGetLastError();
  }
  int lanes = 1;
  while (uint32_t(lanes * kGroupsPerLane) < g.groups) lanes *= 2;
  const uint32_t per_block = uint32_t(kThreads / lanes) * kTokensPerGroup;
  const uint32_t blocks = (g.tokens + per_block - 1) / per_block;
  auto o = static_cast<TOut*>(out);
  auto xi = static_cast<const TIn*>(x);
  switch (lanes) {
    case 1: patch_merge_norm_kernel<TIn, TOut, 1, kGroupsPerLane, kTokensPerGroup><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
    case 2: patch_merge_norm_kernel<TIn, TOut, 2, kGroupsPerLane, kTokensPerGroup><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
    case 4: patch_merge_norm_kernel<TIn, TOut, 4, kGroupsPerLane, kTokensPerGroup><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
    case 8: patch_merge_norm_kernel<TIn, TOut, 8, kGroupsPerLane, kTokensPerGroup><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
    case 16: patch_merge_norm_kernel<TIn, TOut, 16, kGroupsPerLane, kTokensPerGroup><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
    default: patch_merge_norm_kernel<TIn, TOut, 32, kGroupsPerLane, kTokensPerGroup><<<blocks, kThreads, 0, stream>>>(o, xi, gamma, beta, g); break;
  }
  return cudaGetLastError();
}

template <typename TIn>
cudaError_t launch_merge_out(int out_dtype, void* out, const void* x, const float* gamma,
                             const float* beta, const MergeGeom& g, cudaStream_t stream) {
  if (out_dtype == kF32) return launch_merge_t<TIn, float>(out, x, gamma, beta, g, stream);
  if (out_dtype == kF16) return launch_merge_t<TIn, __half>(out, x, gamma, beta, g, stream);
  return launch_merge_t<TIn, __nv_bfloat16>(out, x, gamma, beta, g, stream);
}

}  // namespace

int launch_patch_merge_norm(void* out, int out_dtype, const void* x, int in_dtype,
                            const float* gamma, const float* beta, float eps, int64_t B, int64_t D,
                            int64_t H, int64_t W, int64_t C, const int* parts,
                            cudaStream_t stream) {
  if (B < 0 || D <= 0 || H <= 0 || W <= 0) return set_error(kErrInvalid, "bad volume dims");
  if (C <= 0 || C % 8 != 0 || 8 * C > kMaxMergeC)
    return set_error(kErrUnsupported, "patch_merge_norm_3d needs C a multiple of 8 and 8C <= 3072");
  if (D * H * W >= (int64_t(1) << 31)) return set_error(kErrInvalid, "D*H*W must be below 2^31");
  if (!parts) return set_error(kErrInvalid, "null part table");
  MergeGeom g{};
  g.parts = 0;
  for (int p = 0; p < 8; ++p) {
    if (parts[p] < 0 || parts[p] > 7) return set_error(kErrInvalid, "part codes are 0..7");
    g.parts |= uint32_t(parts[p]) << (3 * p);
  }
  if (B == 0) return kOk;
  if (!out || !x || !gamma || !beta) return set_error(kErrInvalid, "null tensor pointer");
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(x) |
       reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15u)
    return set_error(kErrInvalid, "tensors must be 16-byte aligned");
  g.D = uint32_t(D);
  g.H = uint32_t(H);
  g.W = uint32_t(W);
  g.C = uint32_t(C);
  g.D2 = (g.D + 1) / 2;
  g.H2 = (g.H + 1) / 2;
  g.W2 = (g.W + 1) / 2;
  g.groups = g.C;  // 8C channels in groups of 8
  g.part_groups = g.C / 8;
  g.f_W2 = DivMod32::make(g.W2);
  g.f_H2 = DivMod32::make(g.H2);
  g.f_D2 = DivMod32::make(g.D2);
  g.f_pg = DivMod32::make(g.part_groups);
  g.eps = eps;
  const uint64_t per_batch = uint64_t(g.D2) * g.H2 * g.W2;
  const uint64_t bmax = ((uint64_t(1) << 31) - 1) / per_batch;
  const int64_t in_row = C * dtype_size(in_dtype), out_row = 8 * C * dtype_size(out_dtype);
  for (int64_t b0 = 0; b0 < B; b0 += int64_t(bmax)) {
    const uint64_t nb = uint64_t(B - b0) < bmax ? uint64_t(B - b0) : bmax;
    g.tokens = uint32_t(nb * per_batch);
    const void* xs = static_cast<const uint8_t*>(x) + uint64_t(b0) * D * H * W * in_row;
    void* os = static_cast<uint8_t*>(out) + uint64_t(b0) * per_batch * out_row;
    cudaError_t err;
    if (in_dtype == kF32)
      err = launch_merge_out<float>(out_dtype, os, xs, gamma, beta, g, stream);
    else if (in_dtype == kF16)
      err = launch_merge_out<__half>(out_dtype, os, xs, gamma, beta, g, stream);
    else
      err = launch_merge_out<__nv_bfloat16>(out_dtype, os, xs, gamma, beta, g, stream);
    if (err != cudaSuccess) return set_cuda_error(err, "patch_merge_norm launch");
  }
  return kOk;
}

}  // namespace crumpet
