// (a) Fused momentum + Nesterov + Frobenius norm for every Muon matrix.
// Reference: opendm/optimizer/muon_adamw.py:381-394 (momentum, Nesterov
// blend) and :118-121 (Frobenius normalisation input of the Newton-Schulz).
//
// One pass over the segment table: each 16 Ki-element chunk reads grad
// (bf16/fp32) and exp_avg (fp32) with 128-bit loads, writes exp_avg and the
// direction (rounded to the Newton-Schulz operand type) with 128-bit stores,
// and writes its partial sum of d^2. A second tiny kernel reduces the partials
// of each matrix in a fixed order (deterministic) and produces the input scale
// 1 / max(||d||_F, eps), or 0 for a zero or non-finite norm.

#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace muon {

constexpr int MOM_THREADS = 256;
constexpr int MOM_VEC = 8;
constexpr int MOM_ITERS = 8;
constexpr int64_t MOM_CHUNK = int64_t(MOM_THREADS) * MOM_VEC * MOM_ITERS;  // 16384

int64_t momentum_chunks(int64_t rows, int64_t cols) {
  const int64_t n = rows * cols;
  return n <= 0 ? 0 : (n + MOM_CHUNK - 1) / MOM_CHUNK;
}

__device__ __forceinline__ int find_segment(const muon_momentum_seg* segs, int n_segs, int64_t chunk) {
  int lo = 0, hi = n_segs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (segs[mid].chunk_begin <= chunk)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

struct MomOut {
  float m, d;
};

// exp_avg = momentum * exp_avg + g  (two roundings, as buffer.mul_().add_())
// d = g + momentum * exp_avg        (one fused multiply-add, as add_(alpha=))
__device__ __forceinline__ MomOut mom_op(float g, float m, float mu, bool nesterov) {
  MomOut o;
  o.m = __fadd_rn(__fmul_rn(mu, m), g);
  o.d = nesterov ? __fmaf_rn(mu, o.m, g) : o.m;
  return o;
}

template <int kGradDt, int kDirDt>
__device__ __forceinline__ void load_grad8(const void* grad, int64_t e, float (&g)[8]) {
  if (grad == nullptr) {
#pragma unroll
    for (int i = 0; i < 8; ++i) g[i] = 0.f;
  } else if constexpr (kGradDt == MUON_BF16) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(grad) + e));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      g[2 * i] = f.x;
      g[2 * i + 1] = f.y;
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(grad) + e);
    const float4 a = __ldg(p), b = __ldg(p + 1);
    g[0] = a.x, g[1] = a.y, g[2] = a.z, g[3] = a.w, g[4] = b.x, g[5] = b.y, g[6] = b.z, g[7] = b.w;
  }
}

template <int kDirDt>
__device__ __forceinline__ void store_dir8(void* dir, int64_t e, const float (&d)[8]) {
  if constexpr (kDirDt == MUON_F32) {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(dir) + e);
    p[0] = make_float4(d[0], d[1], d[2], d[3]);
    p[1] = make_float4(d[4], d[5], d[6], d[7]);
  } else if constexpr (kDirDt == MUON_BF16) {
    uint4 raw;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(d[2 * i], d[2 * i + 1]);
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dir) + e) = raw;
  } else {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(dir) + e);
    p[0] = make_float4(round_tf32(d[0]), round_tf32(d[1]), round_tf32(d[2]), round_tf32(d[3]));
    p[1] = make_float4(round_tf32(d[4]), round_tf32(d[5]), round_tf32(d[6]), round_tf32(d[7]));
  }
}

// Gradient-norm clipping folded into the read (clip.cu): g' = g * coef as
// torch's CUDA _foreach_mul_ computes it for a gradient list and a 0-d
// coefficient tensor: the coefficient in the gradient's dtype, the product
// rounded to it.
template <int kGradDt>
__device__ __forceinline__ float clip_grad(float g, float coef) {
  return kGradDt == MUON_BF16 ? bf16_round(g * bf16_round(coef)) : g * coef;
}

template <int kGradDt, int kDirDt>
__global__ void __launch_bounds__(MOM_THREADS) momentum_kernel(const muon_momentum_seg* __restrict__ segs,
                                                               int n_segs, float mu, int nesterov,
                                                               float* __restrict__ partials,
                                                               const float* __restrict__ grad_scale) {
  __shared__ float red[MOM_THREADS / 32];
  const int64_t chunk = blockIdx.x;
  const int s = find_segment(segs, n_segs, chunk);
  const muon_momentum_seg sg = segs[s];
  const int64_t numel = sg.rows * sg.cols;
  const int64_t e0 = (chunk - sg.chunk_begin) * MOM_CHUNK;
  const int64_t e1 = min(e0 + MOM_CHUNK, numel);
  const bool nest = nesterov != 0;
  const bool vec_ok = sg.ld == sg.cols && (numel % 8) == 0 &&
                      ((reinterpret_cast<uintptr_t>(sg.grad) | reinterpret_cast<uintptr_t>(sg.exp_avg) |
                        reinterpret_cast<uintptr_t>(sg.direction)) & 15u) == 0;
  float acc = 0.f;
  if (vec_ok) {
#pragma unroll 2
    for (int it = 0; it < MOM_ITERS; ++it) {
      const int64_t e = e0 + (int64_t(it) * MOM_THREADS + threadIdx.x) * MOM_VEC;
      if (e >= e1) break;
      float g[8];
      load_grad8<kGradDt, kDirDt>(sg.grad, e, g);
      if (grad_scale != nullptr && sg.grad != nullptr) {
        const float coef = *grad_scale;
#pragma unroll
        for (int i = 0; i < 8; ++i) g[i] = clip_grad<kGradDt>(g[i], coef);
      }
      float4* mp = reinterpret_cast<float4*>(sg.exp_avg + e);
      const float4 m0 = mp[0], m1 = mp[1];
      const float mo[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
      float mn[8], d[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const MomOut o = mom_op(g[i], mo[i], mu, nest);
        mn[i] = o.m;
        d[i] = o.d;
        acc = fmaf(o.d, o.d, acc);
      }
      mp[0] = make_float4(mn[0], mn[1], mn[2], mn[3]);
      mp[1] = make_float4(mn[4], mn[5], mn[6], mn[7]);
      if (sg.direction != nullptr) store_dir8<kDirDt>(sg.direction, e, d);
    }
  } else {
    for (int64_t e = e0 + threadIdx.x; e < e1; e += MOM_THREADS) {
      float g = 0.f;
      if (sg.grad) {
        if constexpr (kGradDt == MUON_BF16)
          g = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sg.grad)[e]);
        else
          g = reinterpret_cast<const float*>(sg.grad)[e];
        if (grad_scale != nullptr) g = clip_grad<kGradDt>(g, *grad_scale);
      }
      const MomOut o = mom_op(g, sg.exp_avg[e], mu, nest);
      sg.exp_avg[e] = o.m;
      acc = fmaf(o.d, o.d, acc);
      if (sg.direction == nullptr) continue;
      const int64_t r = e / sg.cols, c = e - r * sg.cols;
      const int64_t di = r * sg.ld + c;
      if constexpr (kDirDt == MUON_BF16)
        reinterpret_cast<__nv_bfloat16*>(sg.direction)[di] = __float2bfloat16_rn(o.d);
      else if constexpr (kDirDt == MUON_F32)
        reinterpret_cast<float*>(sg.direction)[di] = o.d;
      else
        reinterpret_cast<float*>(sg.direction)[di] = round_tf32(o.d);
    }
  }
  // Deterministic block reduction of sum(d^2).
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < MOM_THREADS / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) partials[chunk] = v;
  }
}

// One warp per segment: fixed-order reduction of its chunk partials, then the
// Newton-Schulz input scale (reference muon_adamw.py:118-121).
__global__ void momentum_scale_kernel(const muon_momentum_seg* __restrict__ segs, int n_segs,
                                      int64_t total_chunks, const float* __restrict__ partials, float eps,
                                      float* __restrict__ scales) {
  const int s = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (s >= n_segs) return;
  const int64_t b = segs[s].chunk_begin;
  const int64_t e = (s + 1 < n_segs) ? segs[s + 1].chunk_begin : total_chunks;
  float acc = 0.f;
  for (int64_t c = b + lane; c < e; c += 32) acc += partials[c];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    const float norm = sqrtf(acc);
    scales[s] = (isfinite(norm) && norm > 0.f) ? 1.0f / fmaxf(norm, eps) : 0.f;
  }
}

int launch_momentum(const muon_momentum_seg* segs_dev, int n_segs, int64_t total_chunks, int grad_dtype,
                    int dir_dtype, float momentum, int nesterov, float eps, float* partials_dev,
                    float* scales_dev, const float* grad_scale, cudaStream_t stream) {
  if (n_segs <= 0) return MUON_OK;
  if (!segs_dev || !partials_dev || !scales_dev) return set_error(MUON_ERR_ARG, "null momentum buffer");
  if (grad_dtype != MUON_BF16 && grad_dtype != MUON_F32)
    return set_error(MUON_ERR_ARG, "grad_dtype must be MUON_BF16 or MUON_F32");
  if (dir_dtype != MUON_BF16 && dir_dtype != MUON_TF32 && dir_dtype != MUON_F32)
    return set_error(MUON_ERR_ARG, "dir_dtype must be MUON_BF16, MUON_TF32 or MUON_F32");
  if (total_chunks > 0x7fffffffLL) return set_error(MUON_ERR_ARG, "too many momentum chunks");
  if (total_chunks > 0) {
    const dim3 grid(static_cast<unsigned>(total_chunks));
#define MUON_MOM_LAUNCH(G, D) \
  momentum_kernel<G, D><<<grid, MOM_THREADS, 0, stream>>>(segs_dev, n_segs, momentum, nesterov, partials_dev, \
                                                          grad_scale)
    if (grad_dtype == MUON_BF16) {
      if (dir_dtype == MUON_BF16) MUON_MOM_LAUNCH(MUON_BF16, MUON_BF16);
      else if (dir_dtype == MUON_TF32) MUON_MOM_LAUNCH(MUON_BF16, MUON_TF32);
      else MUON_MOM_LAUNCH(MUON_BF16, MUON_F32);
    } else {
      if (dir_dtype == MUON_BF16) MUON_MOM_LAUNCH(MUON_F32, MUON_BF16);
      else if (dir_dtype == MUON_TF32) MUON_MOM_LAUNCH(MUON_F32, MUON_TF32);
      else MUON_MOM_LAUNCH(MUON_F32, MUON_F32);
    }
#undef MUON_MOM_LAUNCH
    if (check_cuda(cudaGetLastError(), "momentum launch")) return MUON_ERR_CUDA;
  }
  const int warps_per_block = 8;
  const int blocks = (n_segs + warps_per_block - 1) / warps_per_block;
  momentum_scale_kernel<<<blocks, warps_per_block * 32, 0, stream>>>(segs_dev, n_segs, total_chunks, partials_dev,
                                                                      eps, scales_dev);
  if (check_cuda(cudaGetLastError(), "momentum scale launch")) return MUON_ERR_CUDA;
  return MUON_OK;
}

// ===========================================================================
// fp16 Newton-Schulz input in the momentum pass itself (muon_momentum_f16).
//
// The normalisation 1/||d|| is only known once every chunk of a matrix has
// been read, so the fp16 operand is written scaled by a power of two p that
// the previous step's norm of the same matrix chose (entries of typical
// magnitude 1/16: far from fp16's overflow and subnormal ranges while the norm
// moves smoothly from step to step). The exact factor r = (1/||d||) * S0 / p,
// which turns the stored x0 = d * p into the normalised input times the
// operand scale S0, goes to the Newton-Schulz launches as the per-matrix input
// scale (muon_ns_class flag MUON_NS_INPUT_SCALED). One pass reads the
// gradient and the momentum and writes the momentum and the operand: 12 bytes
// per element for bf16 gradients.
//
// A matrix whose p is missing (first step) or no longer safe (the norm moved
// by more than the headroom allows) is rewritten by a fix-up pass with the
// new p; every other chunk of that pass returns at once.
constexpr float kF16Headroom = 1.0f / 16.0f;   // stored entries ~1/16 instead of ~1
constexpr float kF16MaxNormTimesP = 32768.0f;  // ||d|| * p below this: no entry can overflow fp16
constexpr float kF16MinRatio = 1.0f / 256.0f;  // p at least this fraction of the ideal one
constexpr int64_t kFixupCtas = 1184;           // fix-up grid (8 CTAs on each of 148 SMs), grid-stride

__device__ __forceinline__ int find_f16_segment(const muon_momentum_f16_seg* segs, int n_segs, int64_t chunk) {
  int lo = 0, hi = n_segs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (segs[mid].chunk_begin <= chunk)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

// Power of two nearest to x > 0 (in the log domain), 0 for x <= 0 or not finite.
__device__ __forceinline__ float pow2_near(float x) {
  if (!(x > 0.f) || !isfinite(x)) return 0.f;
  int e = 0;
  const float m = frexpf(x, &e);  // x = m * 2^e, m in [0.5, 1)
  return ldexpf(1.0f, m >= 0.70710678f ? e : e - 1);
}

// fp16 operand stores; with lo_offset != 0 (split operands) also the low half
// fp16(x - fp16(x)), lo_offset elements further on.
__device__ __forceinline__ void store_f16x8(__half* dst, int64_t lo_offset, int64_t e, const float (&x)[8]) {
  uint4 hi, lo;
  __half2* h = reinterpret_cast<__half2*>(&hi);
  __half2* l = reinterpret_cast<__half2*>(&lo);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    h[i] = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
    const float2 hf = __half22float2(h[i]);
    l[i] = __floats2half2_rn(x[2 * i] - hf.x, x[2 * i + 1] - hf.y);
  }
  *reinterpret_cast<uint4*>(dst + e) = hi;
  if (lo_offset != 0) *reinterpret_cast<uint4*>(dst + lo_offset + e) = lo;
}

__device__ __forceinline__ void store_f16(__half* dst, int64_t lo_offset, int64_t idx, float x) {
  const __half h = __float2half_rn(x);
  dst[idx] = h;
  if (lo_offset != 0) dst[lo_offset + idx] = __float2half_rn(x - __half2float(h));
}

template <int kGradDt>
__global__ void __launch_bounds__(MOM_THREADS) momentum_f16_kernel(const muon_momentum_f16_seg* __restrict__ segs,
                                                                   int n_segs, float mu, int nesterov,
                                                                   float* __restrict__ partials,
                                                                   const float* __restrict__ pscale,
                                                                   const float* __restrict__ grad_scale) {
  __shared__ float red[MOM_THREADS / 32];
  const int64_t chunk = blockIdx.x;
  const muon_momentum_f16_seg sg = segs[find_f16_segment(segs, n_segs, chunk)];
  const int64_t numel = sg.rows * sg.cols;
  const int64_t e0 = (chunk - sg.chunk_begin) * MOM_CHUNK;
  const int64_t e1 = min(e0 + MOM_CHUNK, numel);
  const bool nest = nesterov != 0;
  const float p = pscale[sg.scale_index];
  const bool write = p > 0.f;  // else the fix-up pass writes this matrix
  const bool clip = grad_scale != nullptr && sg.grad != nullptr;
  const float coef = clip ? *grad_scale : 1.f;
  __half* dst = reinterpret_cast<__half*>(sg.dst);
  const bool vec_ok = sg.ld == sg.cols && (numel % 8) == 0 && (sg.lo_offset % 8) == 0 &&
                      ((reinterpret_cast<uintptr_t>(sg.grad) | reinterpret_cast<uintptr_t>(sg.exp_avg) |
                        reinterpret_cast<uintptr_t>(sg.dst)) & 15u) == 0;
  float acc = 0.f;
  if (vec_ok) {
#pragma unroll 2
    for (int it = 0; it < MOM_ITERS; ++it) {
      const int64_t e = e0 + (int64_t(it) * MOM_THREADS + threadIdx.x) * MOM_VEC;
      if (e >= e1) break;
      float g[8];
      load_grad8<kGradDt, MUON_F16>(sg.grad, e, g);
      if (clip) {
#pragma unroll
        for (int i = 0; i < 8; ++i) g[i] = clip_grad<kGradDt>(g[i], coef);
      }
      float4* mp = reinterpret_cast<float4*>(sg.exp_avg + e);
      const float4 m0 = mp[0], m1 = mp[1];
      const float mo[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
      float mn[8], x[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const MomOut o = mom_op(g[i], mo[i], mu, nest);
        mn[i] = o.m;
        x[i] = o.d * p;  // exact: p is a power of two
        acc = fmaf(o.d, o.d, acc);
      }
      mp[0] = make_float4(mn[0], mn[1], mn[2], mn[3]);
      mp[1] = make_float4(mn[4], mn[5], mn[6], mn[7]);
      if (write) store_f16x8(dst, sg.lo_offset, e, x);
    }
  } else {
    for (int64_t e = e0 + threadIdx.x; e < e1; e += MOM_THREADS) {
      float g = 0.f;
      if (sg.grad) {
        if constexpr (kGradDt == MUON_BF16)
          g = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sg.grad)[e]);
        else
          g = reinterpret_cast<const float*>(sg.grad)[e];
        if (clip) g = clip_grad<kGradDt>(g, coef);
      }
      const MomOut o = mom_op(g, sg.exp_avg[e], mu, nest);
      sg.exp_avg[e] = o.m;
      acc = fmaf(o.d, o.d, acc);
      if (write) store_f16(dst, sg.lo_offset, (e / sg.cols) * sg.ld + e % sg.cols, o.d * p);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < MOM_THREADS / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) partials[chunk] = v;
  }
}

// One warp per segment: the fixed-order norm reduction of momentum_scale_kernel,
// then the Newton-Schulz input factor r, the fix-up decision and the next p.
__global__ void momentum_f16_scale_kernel(const muon_momentum_f16_seg* __restrict__ segs, int n_segs,
                                          int64_t total_chunks, const float* __restrict__ partials, float eps,
                                          float* __restrict__ pscale, float* __restrict__ scales,
                                          int* __restrict__ redo) {
  const int s = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (s >= n_segs) return;
  const int64_t b = segs[s].chunk_begin;
  const int64_t e = (s + 1 < n_segs) ? segs[s + 1].chunk_begin : total_chunks;
  float acc = 0.f;
  for (int64_t c = b + lane; c < e; c += 32) acc += partials[c];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    const int idx = segs[s].scale_index;
    const float norm = sqrtf(acc);
    const float sc = (isfinite(norm) && norm > 0.f) ? 1.0f / fmaxf(norm, eps) : 0.f;
    const float s0 = segs[s].mul;  // operand scale S0 of the first iteration
    const float p_old = pscale[idx];
    if (sc == 0.f) {  // zero or non-finite: the Newton-Schulz result is zero
      scales[idx] = 0.f;
      redo[idx] = 0;
      return;
    }
    const float p_ideal = pow2_near(s0 * sc * kF16Headroom);
    const bool keep = p_old > 0.f && norm * p_old < kF16MaxNormTimesP && p_old >= p_ideal * kF16MinRatio;
    const float p_used = keep ? p_old : p_ideal;
    scales[idx] = sc * s0 / p_used;
    redo[idx] = keep ? 0 : 1;
    if (p_ideal > 0.f) pscale[idx] = p_ideal;  // the next step's p (and the fix-up's)
  }
}

// Fix-up: the operand of the matrices flagged by momentum_f16_scale_kernel,
// rebuilt from the gradient and the advanced momentum with the same
// operations and written as fp16(d * p) with the new p. Every CTA reads the
// flags of 256 segments at a time in one parallel pass and then takes its
// share (grid stride) of the chunks of the flagged ones, so a step without
// fix-ups costs each CTA one or two dependent loads per 256 segments.
template <int kGradDt>
__device__ __forceinline__ void fixup_chunk(const muon_momentum_f16_seg& sg, int64_t chunk, float p, float mu,
                                            bool nest, const float* __restrict__ grad_scale);

template <int kGradDt>
__global__ void __launch_bounds__(MOM_THREADS) momentum_f16_fixup_kernel(const muon_momentum_f16_seg* __restrict__ segs,
                                                                         int n_segs, int64_t total_chunks, float mu,
                                                                         int nesterov,
                                                                         const float* __restrict__ pscale,
                                                                         const int* __restrict__ redo,
                                                                         const float* __restrict__ grad_scale) {
  __shared__ int flagged[MOM_THREADS];
  __shared__ int n_flagged;
  for (int base = 0; base < n_segs; base += MOM_THREADS) {
    if (threadIdx.x == 0) n_flagged = 0;
    __syncthreads();
    const int s = base + static_cast<int>(threadIdx.x);
    if (s < n_segs && redo[segs[s].scale_index] != 0) flagged[atomicAdd(&n_flagged, 1)] = s;
    __syncthreads();
    const int nf = n_flagged;
    for (int f = 0; f < nf; ++f) {
      const int si = flagged[f];
      const muon_momentum_f16_seg sg = segs[si];
      const int64_t end = si + 1 < n_segs ? segs[si + 1].chunk_begin : total_chunks;
      const float p = pscale[sg.scale_index];
      for (int64_t chunk = sg.chunk_begin + blockIdx.x; chunk < end; chunk += gridDim.x)
        fixup_chunk<kGradDt>(sg, chunk, p, mu, nesterov != 0, grad_scale);
    }
    __syncthreads();  // every thread is done with flagged[] before the next batch
  }
}

template <int kGradDt>
__device__ __forceinline__ void fixup_chunk(const muon_momentum_f16_seg& sg, int64_t chunk, float p, float mu,
                                            bool nest, const float* __restrict__ grad_scale) {
  const int64_t numel = sg.rows * sg.cols;
  const int64_t e0 = (chunk - sg.chunk_begin) * MOM_CHUNK;
  const int64_t e1 = min(e0 + MOM_CHUNK, numel);
  const bool clip = grad_scale != nullptr && sg.grad != nullptr;
  const float coef = clip ? *grad_scale : 1.f;
  __half* dst = reinterpret_cast<__half*>(sg.dst);
  const bool vec_ok = sg.ld == sg.cols && (numel % 8) == 0 && (sg.lo_offset % 8) == 0 &&
                      ((reinterpret_cast<uintptr_t>(sg.grad) | reinterpret_cast<uintptr_t>(sg.exp_avg) |
                        reinterpret_cast<uintptr_t>(sg.dst)) & 15u) == 0;
  if (vec_ok) {
    for (int it = 0; it < MOM_ITERS; ++it) {
      const int64_t e = e0 + (int64_t(it) * MOM_THREADS + threadIdx.x) * MOM_VEC;
      if (e >= e1) break;
      float g[8];
      load_grad8<kGradDt, MUON_F16>(sg.grad, e, g);
      const float4* mp = reinterpret_cast<const float4*>(sg.exp_avg + e);
      const float4 m0 = __ldg(mp), m1 = __ldg(mp + 1);
      const float m[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
      float x[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float gi = clip ? clip_grad<kGradDt>(g[i], coef) : g[i];
        x[i] = (nest ? __fmaf_rn(mu, m[i], gi) : m[i]) * p;
      }
      store_f16x8(dst, sg.lo_offset, e, x);
    }
    return;
  }
  for (int64_t e = e0 + threadIdx.x; e < e1; e += MOM_THREADS) {
    float g = 0.f;
    if (sg.grad) {
      if constexpr (kGradDt == MUON_BF16)
        g = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sg.grad)[e]);
      else
        g = reinterpret_cast<const float*>(sg.grad)[e];
      if (clip) g = clip_grad<kGradDt>(g, coef);
    }
    const float m = sg.exp_avg[e];
    const float d = nest ? __fmaf_rn(mu, m, g) : m;
    store_f16(dst, sg.lo_offset, (e / sg.cols) * sg.ld + e % sg.cols, d * p);
  }
}

int launch_momentum_f16(const muon_momentum_f16_seg* segs_dev, int n_segs, int64_t total_chunks, int grad_dtype,
                        float momentum, int nesterov, float eps, float* partials_dev, float* pscale_dev,
                        float* scales_dev, int* redo_dev, const float* grad_scale, cudaStream_t stream) {
  if (n_segs <= 0) return MUON_OK;
  if (!segs_dev || !partials_dev || !pscale_dev || !scales_dev || !redo_dev)
    return set_error(MUON_ERR_ARG, "null momentum_f16 buffer");
  if (grad_dtype != MUON_BF16 && grad_dtype != MUON_F32)
    return set_error(MUON_ERR_ARG, "grad_dtype must be MUON_BF16 or MUON_F32");
  if (total_chunks > 0x7fffffffLL) return set_error(MUON_ERR_ARG, "too many momentum chunks");
  const dim3 grid(static_cast<unsigned>(total_chunks > 0 ? total_chunks : 1));
  if (total_chunks > 0) {
    if (grad_dtype == MUON_BF16)
      momentum_f16_kernel<MUON_BF16><<<grid, MOM_THREADS, 0, stream>>>(segs_dev, n_segs, momentum, nesterov,
                                                                      partials_dev, pscale_dev, grad_scale);
    else
      momentum_f16_kernel<MUON_F32><<<grid, MOM_THREADS, 0, stream>>>(segs_dev, n_segs, momentum, nesterov,
                                                                     partials_dev, pscale_dev, grad_scale);
    if (check_cuda(cudaGetLastError(), "momentum_f16 launch")) return MUON_ERR_CUDA;
  }
  const int warps_per_block = 8;
  momentum_f16_scale_kernel<<<(n_segs + warps_per_block - 1) / warps_per_block, warps_per_block * 32, 0, stream>>>(
      segs_dev, n_segs, total_chunks, partials_dev, eps, pscale_dev, scales_dev, redo_dev);
  if (check_cuda(cudaGetLastError(), "momentum_f16 scale launch")) return MUON_ERR_CUDA;
  if (total_chunks > 0) {
    const dim3 fix_grid(static_cast<unsigned>(total_chunks < kFixupCtas ? total_chunks : kFixupCtas));
    if (grad_dtype == MUON_BF16)
      momentum_f16_fixup_kernel<MUON_BF16><<<fix_grid, MOM_THREADS, 0, stream>>>(
          segs_dev, n_segs, total_chunks, momentum, nesterov, pscale_dev, redo_dev, grad_scale);
    else
      momentum_f16_fixup_kernel<MUON_F32><<<fix_grid, MOM_THREADS, 0, stream>>>(
          segs_dev, n_segs, total_chunks, momentum, nesterov, pscale_dev, redo_dev, grad_scale);
    if (check_cuda(cudaGetLastError(), "momentum_f16 fix-up launch")) return MUON_ERR_CUDA;
  }
  return MUON_OK;
}

// ===========================================================================
// Allocation-free variant for one matrix (muon_momentum_single_noalloc).
//
// Some callers cannot allocate device memory at all: code that runs inside a
// host framework whose memory pool owns every allocation, or inside a region
// where cudaMalloc is forbidden. This variant takes only the caller's inputs
// and outputs; its scratch (one partial sum of d^2 per 16 Ki-element chunk) is
// this file-scope device array, which every GPU that loads the library keeps
// until the process exits. Calls that overlap on the GPU share the array and
// race; each call writes every partial it later reads, so nothing needs to be
// cleared between calls.
constexpr int64_t kNoAllocMaxChunks = 16384;  // 64 KiB: up to 16384 * 16384 elements
constexpr int kMaxNoAllocDevices = 64;

static __device__ __align__(256) float g_noalloc_partials[kNoAllocMaxChunks];

template <int kGradDt, int kDirDt>
__global__ void __launch_bounds__(MOM_THREADS) momentum_single_noalloc_kernel(muon_momentum_seg sg, float mu,
                                                                              int nesterov,
                                                                              float* __restrict__ partials) {
  __shared__ float red[MOM_THREADS / 32];
  const int64_t chunk = blockIdx.x;
  const int64_t numel = sg.rows * sg.cols;
  const int64_t e0 = chunk * MOM_CHUNK;
  const int64_t e1 = min(e0 + MOM_CHUNK, numel);
  const bool nest = nesterov != 0;
  const bool vec_ok = sg.ld == sg.cols && (numel % 8) == 0 &&
                      ((reinterpret_cast<uintptr_t>(sg.grad) | reinterpret_cast<uintptr_t>(sg.exp_avg) |
                        reinterpret_cast<uintptr_t>(sg.direction)) & 15u) == 0;
  float acc = 0.f;
  if (vec_ok) {
    for (int it = 0; it < MOM_ITERS; ++it) {
      const int64_t e = e0 + (int64_t(it) * MOM_THREADS + threadIdx.x) * MOM_VEC;
      if (e >= e1) break;
      float g[8];
      load_grad8<kGradDt, kDirDt>(sg.grad, e, g);
      float4* mp = reinterpret_cast<float4*>(sg.exp_avg + e);
      const float4 m0 = mp[0], m1 = mp[1];
      const float mo[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
      float mn[8], d[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const MomOut o = mom_op(g[i], mo[i], mu, nest);
        mn[i] = o.m;
        d[i] = o.d;
        acc = fmaf(o.d, o.d, acc);
      }
      mp[0] = make_float4(mn[0], mn[1], mn[2], mn[3]);
      mp[1] = make_float4(mn[4], mn[5], mn[6], mn[7]);
      store_dir8<kDirDt>(sg.direction, e, d);
    }
  } else {
    for (int64_t e = e0 + threadIdx.x; e < e1; e += MOM_THREADS) {
      float g = 0.f;
      if (sg.grad) {
        if constexpr (kGradDt == MUON_BF16)
          g = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sg.grad)[e]);
        else
          g = reinterpret_cast<const float*>(sg.grad)[e];
      }
      const MomOut o = mom_op(g, sg.exp_avg[e], mu, nest);
      sg.exp_avg[e] = o.m;
      acc = fmaf(o.d, o.d, acc);
      const int64_t r = e / sg.cols, c = e - r * sg.cols;
      const int64_t di = r * sg.ld + c;
      if constexpr (kDirDt == MUON_BF16)
        reinterpret_cast<__nv_bfloat16*>(sg.direction)[di] = __float2bfloat16_rn(o.d);
      else if constexpr (kDirDt == MUON_F32)
        reinterpret_cast<float*>(sg.direction)[di] = o.d;
      else
        reinterpret_cast<float*>(sg.direction)[di] = round_tf32(o.d);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < MOM_THREADS / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) partials[chunk] = v;
  }
}

// Same fixed-order reduction as momentum_scale_kernel, for one matrix.
__global__ void momentum_single_scale_kernel(const float* __restrict__ partials, int64_t n_chunks, float eps,
                                             float* __restrict__ scale_out) {
  const int lane = threadIdx.x & 31;
  float acc = 0.f;
  for (int64_t c = lane; c < n_chunks; c += 32) acc += partials[c];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    const float norm = sqrtf(acc);
    *scale_out = (isfinite(norm) && norm > 0.f) ? 1.0f / fmaxf(norm, eps) : 0.f;
  }
}

// Device address of g_noalloc_partials, resolved once per device (with that
// device current) on the first call made on it. The address belongs to the
// device's context as it was at that call: after cudaDeviceReset (or anything
// else that destroys the primary context) the library's module is loaded
// again and the cached address is stale, so the entry point must not be used
// in a process that resets a device it has already called it on.
static std::mutex g_noalloc_mutex;
static float* g_noalloc_ptr[kMaxNoAllocDevices] = {};

static int noalloc_scratch(float** out) {
  int dev = 0;
  if (check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return MUON_ERR_CUDA;
  if (dev < 0 || dev >= kMaxNoAllocDevices) return set_error(MUON_ERR_DEVICE, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (check_cuda(cudaGetSymbolAddress(&p, g_noalloc_partials), "cudaGetSymbolAddress(g_noalloc_partials)"))
      return MUON_ERR_CUDA;
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return MUON_OK;
}

int launch_momentum_single_noalloc(const void* grad, float* exp_avg, void* direction, int64_t rows, int64_t cols,
                                   int64_t ld, int grad_dtype, int dir_dtype, float momentum, int nesterov,
                                   float eps, float* scale_out, cudaStream_t stream) {
  if (!exp_avg || !direction || !scale_out) return set_error(MUON_ERR_ARG, "null exp_avg, direction or scale_out");
  if (rows < 0 || cols < 0 || ld < cols) return set_error(MUON_ERR_ARG, "invalid matrix shape or leading dimension");
  if (grad_dtype != MUON_BF16 && grad_dtype != MUON_F32)
    return set_error(MUON_ERR_ARG, "grad_dtype must be MUON_BF16 or MUON_F32");
  if (dir_dtype != MUON_BF16 && dir_dtype != MUON_TF32 && dir_dtype != MUON_F32)
    return set_error(MUON_ERR_ARG, "dir_dtype must be MUON_BF16, MUON_TF32 or MUON_F32");
  // The limit is checked on the factors, before any product is formed, so a
  // shape whose rows * cols (or rows * ld) would overflow int64 is rejected too.
  constexpr int64_t kMaxElements = kNoAllocMaxChunks * MOM_CHUNK;
  static_assert(kMaxElements == MUON_NOALLOC_MAX_ELEMENTS, "limit and header disagree");
  if (rows > 0 && (cols > kMaxElements / rows || ld > kMaxElements / rows)) {
    char msg[200];
    snprintf(msg, sizeof(msg),
             "matrix of %lld x %lld (leading dimension %lld) exceeds the allocation-free limit of %lld elements; "
             "use muon_momentum",
             static_cast<long long>(rows), static_cast<long long>(cols), static_cast<long long>(ld),
             static_cast<long long>(kMaxElements));
    return set_error(MUON_ERR_ARG, msg);
  }
  const int64_t chunks = momentum_chunks(rows, cols);
  float* partials = nullptr;
  const int rc = noalloc_scratch(&partials);
  if (rc != MUON_OK) return rc;
  muon_momentum_seg sg;
  sg.grad = grad;
  sg.exp_avg = exp_avg;
  sg.direction = direction;
  sg.rows = rows;
  sg.cols = cols;
  sg.ld = ld;
  sg.chunk_begin = 0;
  if (chunks > 0) {
    const dim3 grid(static_cast<unsigned>(chunks));
#define MUON_NOALLOC_LAUNCH(G, D) \
  momentum_single_noalloc_kernel<G, D><<<grid, MOM_THREADS, 0, stream>>>(sg, momentum, nesterov, partials)
    if (grad_dtype == MUON_BF16) {
      if (dir_dtype == MUON_BF16) MUON_NOALLOC_LAUNCH(MUON_BF16, MUON_BF16);
      else if (dir_dtype == MUON_TF32) MUON_NOALLOC_LAUNCH(MUON_BF16, MUON_TF32);
      else MUON_NOALLOC_LAUNCH(MUON_BF16, MUON_F32);
    } else {
      if (dir_dtype == MUON_BF16) MUON_NOALLOC_LAUNCH(MUON_F32, MUON_BF16);
      else if (dir_dtype == MUON_TF32) MUON_NOALLOC_LAUNCH(MUON_F32, MUON_TF32);
      else MUON_NOALLOC_LAUNCH(MUON_F32, MUON_F32);
    }
#undef MUON_NOALLOC_LAUNCH
    if (check_cuda(cudaGetLastError(), "momentum (no-alloc) launch")) return MUON_ERR_CUDA;
  }
  momentum_single_scale_kernel<<<1, 32, 0, stream>>>(partials, chunks, eps, scale_out);
  if (check_cuda(cudaGetLastError(), "momentum scale (no-alloc) launch")) return MUON_ERR_CUDA;
  return MUON_OK;
}

}  // namespace muon
