// Fused AdamW for the reference's non-Muon parameter group.
// Reference: _adamw_step / _call_adamw_functional (opendm/optimizer/
// muon_adamw.py:131-175, :333-343), which calls torch.optim.adamw's
// single-tensor path (decoupled weight decay) once per parameter. Here every
// parameter of the group is one segment of a single launch and each element
// is read and written once:
//   p = p * (1 - lr*wd)                      (rounded to the param dtype)
//   m = m + (1 - beta1) * (g - m)            (lerp, fused multiply-add)
//   v = fl(v * beta2) + fl(fl((1-beta2) * g) * g)
//   p = p + (-step_size) * (m / (fl(sqrt(v) / bc2_sqrt) + eps))
// The rounding sequence follows torch's CPU kernels for these ops.

#include "common.cuh"
#include "internal.h"

namespace muon {

constexpr int ADAM_THREADS = 256;
constexpr int ADAM_VEC = 4;
constexpr int ADAM_ITERS = 8;
constexpr int64_t ADAM_CHUNK = int64_t(ADAM_THREADS) * ADAM_VEC * ADAM_ITERS;  // 8192

int64_t adamw_chunks(int64_t numel) { return numel <= 0 ? 0 : (numel + ADAM_CHUNK - 1) / ADAM_CHUNK; }

__device__ __forceinline__ int find_adam_segment(const muon_adamw_seg* segs, int n_segs, int64_t chunk) {
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

__device__ __forceinline__ float adam_elem(float p, float g, float& m, float& v, float beta1w, float beta2,
                                           float one_minus_beta2, float eps, float wd_factor, float neg_step,
                                           float bc2_sqrt, bool bf16_param) {
  if (wd_factor != 1.f) {
    p = p * wd_factor;
    if (bf16_param) p = bf16_round(p);
  }
  m = fmaf(beta1w, g - m, m);
  v = __fadd_rn(__fmul_rn(v, beta2), __fmul_rn(__fmul_rn(one_minus_beta2, g), g));
  const float denom = __fadd_rn(__fdiv_rn(sqrtf(v), bc2_sqrt), eps);
  return __fadd_rn(p, __fmul_rn(neg_step, __fdiv_rn(m, denom)));
}

// Gradient-norm clipping folded into the read (clip.cu): g' = g * coef with
// the coefficient and the product in the gradient's dtype (torch's CUDA
// _foreach_mul_ with a 0-d coefficient tensor).
__device__ __forceinline__ float clip_grad_adam(float g, float coef, bool bf) {
  return bf ? bf16_round(g * bf16_round(coef)) : g * coef;
}

__global__ void __launch_bounds__(ADAM_THREADS) adamw_kernel(const muon_adamw_seg* __restrict__ segs, int n_segs,
                                                             float beta1w, float beta2, float one_minus_beta2,
                                                             float eps, float wd_factor,
                                                             const float* __restrict__ grad_scale) {
  const int64_t chunk = blockIdx.x;
  const muon_adamw_seg sg = segs[find_adam_segment(segs, n_segs, chunk)];
  const int64_t e0 = (chunk - sg.chunk_begin) * ADAM_CHUNK;
  const int64_t e1 = min(e0 + ADAM_CHUNK, sg.numel);
  const bool pbf = sg.param_dtype == MUON_BF16;
  const bool gbf = sg.grad_dtype == MUON_BF16;
  const float neg_step = -sg.step_size;
  const bool vec_ok = (sg.numel % 4) == 0 &&
                      ((reinterpret_cast<uintptr_t>(sg.param) | reinterpret_cast<uintptr_t>(sg.grad) |
                        reinterpret_cast<uintptr_t>(sg.exp_avg) | reinterpret_cast<uintptr_t>(sg.exp_avg_sq)) &
                       15u) == 0;
  if (vec_ok) {
    for (int it = 0; it < ADAM_ITERS; ++it) {
      const int64_t e = e0 + (int64_t(it) * ADAM_THREADS + threadIdx.x) * ADAM_VEC;
      if (e >= e1) break;
      float p[4], g[4];
      if (pbf) {
        const uint2 raw = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(sg.param) + e);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
        const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
        p[0] = a.x, p[1] = a.y, p[2] = b.x, p[3] = b.y;
      } else {
        const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(sg.param) + e);
        p[0] = a.x, p[1] = a.y, p[2] = a.z, p[3] = a.w;
      }
      if (gbf) {
        const uint2 raw = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(sg.grad) + e));
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
        const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
        g[0] = a.x, g[1] = a.y, g[2] = b.x, g[3] = b.y;
      } else {
        const float4 a = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(sg.grad) + e));
        g[0] = a.x, g[1] = a.y, g[2] = a.z, g[3] = a.w;
      }
      if (grad_scale != nullptr) {
        const float coef = *grad_scale;
#pragma unroll
        for (int i = 0; i < 4; ++i) g[i] = clip_grad_adam(g[i], coef, gbf);
      }
      float4 m4 = *reinterpret_cast<float4*>(sg.exp_avg + e);
      float4 v4 = *reinterpret_cast<float4*>(sg.exp_avg_sq + e);
      float m[4] = {m4.x, m4.y, m4.z, m4.w}, v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        p[i] = adam_elem(p[i], g[i], m[i], v[i], beta1w, beta2, one_minus_beta2, eps, wd_factor, neg_step,
                         sg.bc2_sqrt, pbf);
      *reinterpret_cast<float4*>(sg.exp_avg + e) = make_float4(m[0], m[1], m[2], m[3]);
      *reinterpret_cast<float4*>(sg.exp_avg_sq + e) = make_float4(v[0], v[1], v[2], v[3]);
      if (pbf) {
        uint2 raw;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
        h[0] = __floats2bfloat162_rn(p[0], p[1]);
        h[1] = __floats2bfloat162_rn(p[2], p[3]);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(sg.param) + e) = raw;
      } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(sg.param) + e) = make_float4(p[0], p[1], p[2], p[3]);
      }
    }
  } else {
    for (int64_t e = e0 + threadIdx.x; e < e1; e += ADAM_THREADS) {
      float p = pbf ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sg.param)[e])
                    : reinterpret_cast<const float*>(sg.param)[e];
      float g = gbf ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sg.grad)[e])
                    : reinterpret_cast<const float*>(sg.grad)[e];
      if (grad_scale != nullptr) g = clip_grad_adam(g, *grad_scale, gbf);
      float m = sg.exp_avg[e], v = sg.exp_avg_sq[e];
      p = adam_elem(p, g, m, v, beta1w, beta2, one_minus_beta2, eps, wd_factor, neg_step, sg.bc2_sqrt, pbf);
      sg.exp_avg[e] = m;
      sg.exp_avg_sq[e] = v;
      if (pbf)
        reinterpret_cast<__nv_bfloat16*>(sg.param)[e] = __float2bfloat16_rn(p);
      else
        reinterpret_cast<float*>(sg.param)[e] = p;
    }
  }
}

int launch_adamw(const muon_adamw_seg* segs_dev, int n_segs, int64_t total_chunks, double beta1, double beta2,
                 float eps, float wd_factor, const float* grad_scale, cudaStream_t stream) {
  if (n_segs <= 0 || total_chunks <= 0) return MUON_OK;
  if (!segs_dev) return set_error(MUON_ERR_ARG, "null AdamW segment table");
  if (total_chunks > 0x7fffffffLL) return set_error(MUON_ERR_ARG, "too many AdamW chunks");
  // (1 - beta1) and (1 - beta2) are formed in double by the reference's
  // Python code and rounded to float when applied.
  const float beta1w = static_cast<float>(1.0 - beta1);
  const float omb2 = static_cast<float>(1.0 - beta2);
  adamw_kernel<<<static_cast<unsigned>(total_chunks), ADAM_THREADS, 0, stream>>>(segs_dev, n_segs, beta1w,
                                                                                 static_cast<float>(beta2), omb2, eps, wd_factor,
                                                                                 grad_scale);
  if (check_cuda(cudaGetLastError(), "adamw launch")) return MUON_ERR_CUDA;
  return MUON_OK;
}

}  // namespace muon
