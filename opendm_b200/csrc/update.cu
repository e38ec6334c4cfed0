// (c) Weight decay + scaled Muon update, one pass per element.
// Reference: opendm/optimizer/muon_adamw.py:395-398 (param.mul_(1 - lr*wd))
// and :407-414 (param.add_(update.to(param.dtype), alpha=-eff)), with the
// same rounding order: the weight-decayed parameter is rounded to the
// parameter dtype, then p + (-eff) * u is one fused multiply-add rounded to
// the parameter dtype. u arrives already rounded to the parameter dtype (the
// last Newton-Schulz epilogue writes it that way).

#include "common.cuh"
#include "internal.h"

namespace muon {

constexpr int UPD_THREADS = 256;
constexpr int UPD_VEC = 8;
constexpr int UPD_ITERS = 8;
constexpr int64_t UPD_CHUNK = int64_t(UPD_THREADS) * UPD_VEC * UPD_ITERS;  // == momentum chunk (16384)

__device__ __forceinline__ int find_update_segment(const muon_update_seg* segs, int n_segs, int64_t chunk) {
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

template <bool kBf16>
__device__ __forceinline__ float upd_elem(float p, float u, float neg_eff, float wd_factor) {
  if (wd_factor != 1.f) p = kBf16 ? bf16_round(p * wd_factor) : p * wd_factor;
  return fmaf(neg_eff, u, p);
}

template <bool kBf16>
__device__ __forceinline__ void update_chunk(const muon_update_seg& sg, int64_t e0, int64_t e1, float wd_factor) {
  const float neg_eff = -sg.eff;
  const int64_t numel = sg.rows * sg.cols;
  const bool vec_ok = sg.ld == sg.cols && (numel % 8) == 0 &&
                      ((reinterpret_cast<uintptr_t>(sg.param) | reinterpret_cast<uintptr_t>(sg.update)) & 15u) == 0;
  if (vec_ok) {
    for (int it = 0; it < UPD_ITERS; ++it) {
      const int64_t e = e0 + (int64_t(it) * UPD_THREADS + threadIdx.x) * UPD_VEC;
      if (e >= e1) break;
      if constexpr (kBf16) {
        uint4* pp = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(sg.param) + e);
        const uint4 praw = *pp;
        const uint4 uraw = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(sg.update) + e));
        const __nv_bfloat162* ph = reinterpret_cast<const __nv_bfloat162*>(&praw);
        const __nv_bfloat162* uh = reinterpret_cast<const __nv_bfloat162*>(&uraw);
        uint4 out;
        __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 p2 = __bfloat1622float2(ph[i]);
          const float2 u2 = __bfloat1622float2(uh[i]);
          oh[i] = __floats2bfloat162_rn(upd_elem<true>(p2.x, u2.x, neg_eff, wd_factor),
                                        upd_elem<true>(p2.y, u2.y, neg_eff, wd_factor));
        }
        *pp = out;
      } else {
        float4* pp = reinterpret_cast<float4*>(reinterpret_cast<float*>(sg.param) + e);
        const float4* up = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(sg.update) + e);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float4 p = pp[h];
          const float4 u = __ldg(up + h);
          p.x = upd_elem<false>(p.x, u.x, neg_eff, wd_factor);
          p.y = upd_elem<false>(p.y, u.y, neg_eff, wd_factor);
          p.z = upd_elem<false>(p.z, u.z, neg_eff, wd_factor);
          p.w = upd_elem<false>(p.w, u.w, neg_eff, wd_factor);
          pp[h] = p;
        }
      }
    }
  } else {
    for (int64_t e = e0 + threadIdx.x; e < e1; e += UPD_THREADS) {
      const int64_t r = e / sg.cols, c = e - r * sg.cols;
      const int64_t ui = r * sg.ld + c;
      if constexpr (kBf16) {
        __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(sg.param) + e;
        const float u = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sg.update)[ui]);
        *p = __float2bfloat16_rn(upd_elem<true>(__bfloat162float(*p), u, neg_eff, wd_factor));
      } else {
        float* p = reinterpret_cast<float*>(sg.param) + e;
        *p = upd_elem<false>(*p, reinterpret_cast<const float*>(sg.update)[ui], neg_eff, wd_factor);
      }
    }
  }
}

__global__ void __launch_bounds__(UPD_THREADS) apply_update_kernel(const muon_update_seg* __restrict__ segs,
                                                                   int n_segs, float wd_factor) {
  const int64_t chunk = blockIdx.x;
  const muon_update_seg sg = segs[find_update_segment(segs, n_segs, chunk)];
  const int64_t e0 = (chunk - sg.chunk_begin) * UPD_CHUNK;
  const int64_t e1 = min(e0 + UPD_CHUNK, sg.rows * sg.cols);
  if (sg.param_dtype == MUON_BF16)
    update_chunk<true>(sg, e0, e1, wd_factor);
  else
    update_chunk<false>(sg, e0, e1, wd_factor);
}

int launch_apply_update(const muon_update_seg* segs_dev, int n_segs, int64_t total_chunks, float wd_factor,
                        cudaStream_t stream) {
  if (n_segs <= 0 || total_chunks <= 0) return MUON_OK;
  if (!segs_dev) return set_error(MUON_ERR_ARG, "null update segment table");
  if (total_chunks > 0x7fffffffLL) return set_error(MUON_ERR_ARG, "too many update chunks");
  apply_update_kernel<<<static_cast<unsigned>(total_chunks), UPD_THREADS, 0, stream>>>(segs_dev, n_segs, wd_factor);
  if (check_cuda(cudaGetLastError(), "apply_update launch")) return MUON_ERR_CUDA;
  return MUON_OK;
}

}  // namespace muon
