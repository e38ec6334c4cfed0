// Gradient-norm clipping folded into the optimizer step.
//
// The reference's trainer clips gradients before every optimizer step
// (opendm/trainer/trainer.py:213, max_grad_norm=1.0) with
// torch.nn.utils.clip_grad_norm_ (torch 2.11.0, torch/nn/utils/clip_grad.py),
// which reads every gradient twice (norms, then an in-place multiply) and
// writes it once. Here the norm pass stays and the multiply moves into the
// momentum and AdamW kernels (muon_momentum_scaled / muon_adamw_scaled),
// which scale each gradient as they read it: one full read and write of the
// gradients fewer. The arithmetic follows torch's, norm type 2:
//   norm_i = round_{dtype_i}(sqrt(sum g^2))           (_foreach_norm)
//   total  = round_{R}(sqrt(sum norm_i^2))            (vector_norm of the stack)
//   coef   = min(round_R(round_R(1 / round_R(total + 1e-6)) * max_norm), 1)
//                                                     (max_norm / t is t.reciprocal() * max_norm)
//   g'     = round_{dtype_i}(g * round_{dtype_i}(coef))  (CUDA _foreach_mul_ with a
//                                                     0-d tensor: the coefficient in the list's dtype)
// with R = bf16 when every gradient is bf16, else fp32. Sums accumulate in
// fp32 in a fixed order (deterministic; torch's own order can differ in the
// last fp32 bit).

#include "common.cuh"
#include "internal.h"

namespace muon {

constexpr int NRM_THREADS = 256;
constexpr int NRM_VEC = 8;
constexpr int NRM_ITERS = 8;
constexpr int64_t NRM_CHUNK = int64_t(NRM_THREADS) * NRM_VEC * NRM_ITERS;  // 16384

int64_t norm_chunks(int64_t numel) { return numel <= 0 ? 0 : (numel + NRM_CHUNK - 1) / NRM_CHUNK; }

__device__ __forceinline__ int find_norm_segment(const muon_norm_seg* segs, int n_segs, int64_t chunk) {
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

__global__ void __launch_bounds__(NRM_THREADS) grad_sumsq_kernel(const muon_norm_seg* __restrict__ segs, int n_segs,
                                                                 float* __restrict__ partials) {
  __shared__ float red[NRM_THREADS / 32];
  const int64_t chunk = blockIdx.x;
  const muon_norm_seg sg = segs[find_norm_segment(segs, n_segs, chunk)];
  const int64_t e0 = (chunk - sg.chunk_begin) * NRM_CHUNK;
  const int64_t e1 = min(e0 + NRM_CHUNK, sg.numel);
  const bool bf = sg.dtype == MUON_BF16;
  const bool vec_ok = (sg.numel % 8) == 0 && (reinterpret_cast<uintptr_t>(sg.grad) & 15u) == 0;
  float acc = 0.f;
  if (vec_ok) {
    for (int it = 0; it < NRM_ITERS; ++it) {
      const int64_t e = e0 + (int64_t(it) * NRM_THREADS + threadIdx.x) * NRM_VEC;
      if (e >= e1) break;
      if (bf) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(sg.grad) + e));
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h[i]);
          acc = fmaf(f.x, f.x, acc);
          acc = fmaf(f.y, f.y, acc);
        }
      } else {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(sg.grad) + e);
        const float4 a = __ldg(p), b = __ldg(p + 1);
        acc = fmaf(a.x, a.x, acc), acc = fmaf(a.y, a.y, acc), acc = fmaf(a.z, a.z, acc), acc = fmaf(a.w, a.w, acc);
        acc = fmaf(b.x, b.x, acc), acc = fmaf(b.y, b.y, acc), acc = fmaf(b.z, b.z, acc), acc = fmaf(b.w, b.w, acc);
      }
    }
  } else {
    for (int64_t e = e0 + threadIdx.x; e < e1; e += NRM_THREADS) {
      const float g = bf ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sg.grad)[e])
                         : reinterpret_cast<const float*>(sg.grad)[e];
      acc = fmaf(g, g, acc);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < NRM_THREADS / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) partials[chunk] = v;
  }
}

__device__ __forceinline__ float round_dt(float x, bool bf) { return bf ? bf16_round(x) : x; }

// One block: a warp per segment sums its chunk partials (lane-strided, then a
// fixed shuffle tree), rounds the norm to the segment's dtype and adds its
// square to the warp's total; the warps' totals are then added in warp order.
// Deterministic. out[0] = total, out[1] = coefficient.
__global__ void __launch_bounds__(NRM_THREADS) clip_coef_kernel(const muon_norm_seg* __restrict__ segs, int n_segs,
                                                                int64_t total_chunks,
                                                                const float* __restrict__ partials, float max_norm,
                                                                float* __restrict__ out) {
  constexpr int kWarps = NRM_THREADS / 32;
  __shared__ float red[kWarps];
  __shared__ int not_bf[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float acc = 0.f;  // sum of squared norms of this warp's segments (lane 0)
  int any_f32 = 0;
  for (int s = warp; s < n_segs; s += kWarps) {
    const int64_t b = segs[s].chunk_begin;
    const int64_t e = (s + 1 < n_segs) ? segs[s + 1].chunk_begin : total_chunks;
    float sum = 0.f;
    for (int64_t c = b + lane; c < e; c += 32) sum += partials[c];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const bool bf = segs[s].dtype == MUON_BF16;
    any_f32 |= bf ? 0 : 1;
    const float norm = round_dt(sqrtf(sum), bf);
    acc = fmaf(norm, norm, acc);
  }
  if (lane == 0) {
    red[warp] = acc;
    not_bf[warp] = any_f32;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = 0.f;
    int f32 = 0;
    for (int w = 0; w < kWarps; ++w) {
      v += red[w];
      f32 |= not_bf[w];
    }
    const bool bf = f32 == 0;
    const float total = round_dt(sqrtf(v), bf);
    const float denom = round_dt(total + 1e-6f, bf);
    const float recip = round_dt(1.0f / denom, bf);
    const float coef = round_dt(recip * max_norm, bf);
    out[0] = total;
    out[1] = (coef != coef) ? coef : fminf(coef, 1.0f);  // a NaN stays NaN, as in torch's clamp
  }
}

int launch_clip_grad_norm(const muon_norm_seg* segs_dev, int n_segs, int64_t total_chunks, float max_norm,
                          float* partials_dev, float* out_dev, cudaStream_t stream) {
  if (!out_dev) return set_error(MUON_ERR_ARG, "null clip output");
  if (n_segs < 0) return set_error(MUON_ERR_ARG, "negative segment count");
  if (n_segs > 0 && (!segs_dev || (total_chunks > 0 && !partials_dev)))
    return set_error(MUON_ERR_ARG, "null norm segment table or partials");
  if (total_chunks > 0x7fffffffLL) return set_error(MUON_ERR_ARG, "too many norm chunks");
  if (n_segs > 0 && total_chunks > 0) {
    grad_sumsq_kernel<<<static_cast<unsigned>(total_chunks), NRM_THREADS, 0, stream>>>(segs_dev, n_segs,
                                                                                       partials_dev);
    if (check_cuda(cudaGetLastError(), "grad_sumsq launch")) return MUON_ERR_CUDA;
  }
  clip_coef_kernel<<<1, NRM_THREADS, 0, stream>>>(segs_dev, n_segs, total_chunks, partials_dev, max_norm, out_dev);
  return check_cuda(cudaGetLastError(), "clip_coef launch");
}

}  // namespace muon
