// Grouped tcgen05/TMEM GEMMs for the Newton-Schulz orthogonalisation
// (reference: zeropower_via_newtonschulz5, opendm/optimizer/muon_adamw.py:101-128).
//
// One launch evaluates one phase of one Newton-Schulz iteration for every
// matrix of every shape class:
//   phase 0 (gram):  A' = s^2 X X^T - I               symmetric m x m, K = n
//   phase 1 (poly):  M  = alpha I + beta A' + gamma A'A'  symmetric m x m, K = m
//   phase 2 (apply): X  = s M X   (wide)  |  X = s X M  (tall: X kept as the
//                    parameter's n x m layout, which is the transpose)
// s is the per-matrix Frobenius scale on the first iteration and 1 after it.
// The last apply either writes the fp32 update U or applies the fused
// weight-decay + scaled update to the parameters
// (reference: muon_adamw.py:395-398, :407-414).
//
// Kernel structure (one CTA per SM, persistent, static round-robin tiles):
//   warp 0      TMA producer: 128B-swizzled operand tiles into a 4-stage ring
//   warp 1      TMEM owner and single-thread tcgen05.mma issuer
//   warps 2..5  epilogue: tcgen05.ld -> registers -> smem transpose ->
//               coalesced global stores (+ mirrored stores for symmetric C)
// Accumulators: two 128 x 256 fp32 buffers in TMEM (all 512 columns), so the
// epilogue of tile i overlaps the main loop of tile i+1.
// Operands are bf16 (kind::f16) or tf32 (kind::tf32); either way a stage
// holds 128 bytes of K per row, so the byte geometry is identical.

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace muon {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int A_STAGE_BYTES = BM * 128;
constexpr int B_STAGE_BYTES = BN * 128;
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int EPI_WARPS = 4;
constexpr int NUM_THREADS = 64 + EPI_WARPS * 32;
constexpr int EPI_PITCH = 33;  // floats per staged row (conflict-free transpose)
constexpr int EPI_BYTES = EPI_WARPS * 32 * EPI_PITCH * 4;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
constexpr int TMEM_COLS = 2 * BN;
constexpr int kMaxProblems = 16;

enum EpiKind : int { EPI_GRAM = 0, EPI_POLY = 1, EPI_APPLY = 2, EPI_APPLY_F32 = 3, EPI_UPDATE = 4 };

// Newton-Schulz quintic coefficients of the reference (muon_adamw.py:123) and
// the shifted-form coefficients derived from them.
constexpr double kNsA = 3.4445, kNsB = -4.7750, kNsC = 2.0315;

struct GemmProblem {
  int M, N, K;
  int batch;
  int tiles_m, tiles_n;
  int tiles_per_mat;
  int tile_begin;
  int a_mn, b_mn;  // operand majorness: 0 = K-major, 1 = MN-major
  int symmetric;   // compute upper-triangle tiles and mirror them
  int epi;
  int first;       // apply the per-matrix input scale
  int param_dtype;
  float eff;
  float wd_factor;
  void* out;
  long long out_ld, out_bs;
  const void* side;
  long long side_ld, side_bs;
  const float* scale;
  void* const* params;
};

struct GemmParams {
  CUtensorMap map_a[kMaxProblems];
  CUtensorMap map_b[kMaxProblems];
  GemmProblem prob[kMaxProblems];
  int n_problems;
  int total_tiles;
  float alpha, beta, gamma;
  int* err;
};

struct TileCoord {
  int p, g, ti, tj;
};

__device__ __forceinline__ TileCoord decode_tile(const GemmParams& P, int t) {
  TileCoord c;
  int p = 0;
  while (p + 1 < P.n_problems && t >= P.prob[p + 1].tile_begin) ++p;
  const GemmProblem& pr = P.prob[p];
  int local = t - pr.tile_begin;
  c.p = p;
  c.g = local / pr.tiles_per_mat;
  int lt = local - c.g * pr.tiles_per_mat;
  if (!pr.symmetric) {
    c.ti = lt / pr.tiles_n;
    c.tj = lt - c.ti * pr.tiles_n;
  } else {
    // Row block ti holds column blocks [ti/2, tiles_n): exactly the tiles that
    // contain an element with col >= row.
    int ti = 0;
    while (true) {
      const int cnt = pr.tiles_n - (ti >> 1);
      if (lt < cnt) {
        c.tj = (ti >> 1) + lt;
        break;
      }
      lt -= cnt;
      ++ti;
    }
    c.ti = ti;
  }
  return c;
}

template <bool kTf32>
__device__ __forceinline__ void store_op(void* base, long long idx, float v) {
  if constexpr (kTf32) {
    reinterpret_cast<float*>(base)[idx] = v;
  } else {
    reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
  }
}

template <bool kTf32>
__device__ __forceinline__ float round_op(float v) {
  if constexpr (kTf32) {
    return round_tf32(v);
  } else {
    return bf16_round(v);
  }
}

template <bool kTf32>
__device__ __forceinline__ float load_op(const void* base, long long idx) {
  if constexpr (kTf32) {
    return reinterpret_cast<const float*>(base)[idx];
  } else {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
  }
}

template <bool kTf32>
__global__ void __launch_bounds__(NUM_THREADS, 1) ns_gemm_kernel(const __grid_constant__ GemmParams P) {
  constexpr int ES = kTf32 ? 4 : 2;
  constexpr int BKE = 128 / ES;     // K elements per stage == MN elements per swizzle atom
  constexpr int UMMA_K = 32 / ES;   // K elements per tcgen05.mma
  constexpr int KSTEPS = BKE / UMMA_K;
  // MN-major operands: bf16 uses the 128B swizzle (8-row K groups, SBO 1024);
  // tf32 must use the 32-byte-atom 128B swizzle (4-row K groups, SBO 512).
  constexpr uint32_t kMnLayout = kTf32 ? kLayoutSw128Base32 : kLayoutSw128;
  constexpr uint32_t kMnSbo = kTf32 ? 512 : 1024;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stage_a = smem;
  uint8_t* stage_b = smem + STAGES * A_STAGE_BYTES;
  float* epi_buf = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES + EPI_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPI_WARPS);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    for (int p = 0; p < P.n_problems; ++p) {
      tma_prefetch_desc(&P.map_a[p]);
      tma_prefetch_desc(&P.map_b[p]);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued[STAGES];
      uint32_t issued_phase[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = 0, issued_phase[s] = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < P.total_tiles; t += gridDim.x) {
        const TileCoord tc = decode_tile(P, t);
        const GemmProblem& pr = P.prob[tc.p];
        const int kb_count = (pr.K + BKE - 1) / BKE;
        const int m0 = tc.ti * BM, n0 = tc.tj * BN;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, P.err, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* sa = stage_a + stage * A_STAGE_BYTES;
          uint8_t* sb = stage_b + stage * B_STAGE_BYTES;
          const int k0 = kb * BKE;
          if (!pr.a_mn) {
            tma_load_3d(sa, &P.map_a[tc.p], &full[stage], k0, m0, tc.g);
          } else {
#pragma unroll
            for (int j = 0; j < BM / BKE; ++j)
              tma_load_3d(sa + j * BKE * 128, &P.map_a[tc.p], &full[stage], m0 + j * BKE, k0, tc.g);
          }
          if (!pr.b_mn) {
            tma_load_3d(sb, &P.map_b[tc.p], &full[stage], k0, n0, tc.g);
          } else {
#pragma unroll
            for (int j = 0; j < BN / BKE; ++j)
              tma_load_3d(sb + j * BKE * 128, &P.map_b[tc.p], &full[stage], n0 + j * BKE, k0, tc.g);
          }
          issued[stage] = 1;
          issued_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: every issued TMA load must have landed before the CTA exits.
      for (int s = 0; s < STAGES; ++s)
        if (issued[s]) mbar_wait(&full[s], issued_phase[s], P.err, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local_t = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < P.total_tiles; t += gridDim.x, ++local_t) {
        const TileCoord tc = decode_tile(P, t);
        const GemmProblem& pr = P.prob[tc.p];
        const int kb_count = (pr.K + BKE - 1) / BKE;
        const int acc = local_t & 1;
        const uint32_t acc_phase = (local_t >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, P.err, kDevTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const uint32_t idesc = make_idesc(kTf32, BM, BN, pr.a_mn != 0, pr.b_mn != 0);
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(&full[stage], phase, P.err, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stage_a + stage * A_STAGE_BYTES);
          const uint32_t b_addr = smem_u32(stage_b + stage * B_STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < KSTEPS; ++kk) {
            const uint64_t ad = pr.a_mn ? make_sw128_desc(a_addr + kk * UMMA_K * 128, BKE * 128, kMnSbo, kMnLayout)
                                        : make_sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = pr.b_mn ? make_sw128_desc(b_addr + kk * UMMA_K * 128, BKE * 128, kMnSbo, kMnLayout)
                                        : make_sw128_desc(b_addr + kk * 32, 16, 1024);
            umma<kTf32>(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      // Drain: all issued MMAs complete before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, P.err, kDevTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    float* buf = epi_buf + (warp - 2) * 32 * EPI_PITCH;
    int local_t = 0;
    for (int t = blockIdx.x; t < P.total_tiles; t += gridDim.x, ++local_t) {
      const TileCoord tc = decode_tile(P, t);
      const GemmProblem& pr = P.prob[tc.p];
      const int acc = local_t & 1;
      const uint32_t acc_phase = (local_t >> 1) & 1;
      // Every lane waits; the outcome is made warp-uniform before the
      // warp-synchronous tcgen05.ld below.
      const bool ready = mbar_wait(&tfull[acc], acc_phase, P.err, kDevTimeoutTmemFull);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();

      float sc = 1.f;
      bool zero = false;
      if (pr.first) {
        sc = pr.scale[tc.g];
        zero = !(sc != 0.f);
      }
      const int row0 = tc.ti * BM + quad * 32;
      const long long out_off = static_cast<long long>(tc.g) * pr.out_bs;
      const long long side_off = static_cast<long long>(tc.g) * pr.side_bs;
      void* param_ptr = (pr.epi == EPI_UPDATE) ? pr.params[tc.g] : nullptr;

      for (int ch = 0; ch < BN / 32; ++ch) {
        const int col0 = tc.tj * BN + ch * 32;
        float v[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN + ch * 32, v);
        if (row0 >= pr.M || col0 >= pr.N) continue;
        if (pr.symmetric && col0 + 31 < row0) continue;  // chunk entirely below the diagonal
#pragma unroll
        for (int i = 0; i < 32; ++i) buf[lane * EPI_PITCH + i] = v[i];
        __syncwarp();
        // Column mode: lane = column, walk the 32 rows (coalesced I/O).
        const int col = col0 + lane;
        for (int r = 0; r < 32; ++r) {
          const int row = row0 + r;
          if (row >= pr.M || col >= pr.N) continue;
          if (pr.symmetric && col < row) continue;
          const float a = buf[r * EPI_PITCH + lane];
          const long long idx = static_cast<long long>(row) * pr.out_ld + col;
          float res;
          switch (pr.epi) {
            case EPI_GRAM: {
              float x = zero ? 0.f : (pr.first ? (sc * sc) * a : a);
              if (row == col) x -= 1.f;
              res = round_op<kTf32>(x);
              store_op<kTf32>(pr.out, out_off + idx, res);
              break;
            }
            case EPI_POLY: {
              const float s = load_op<kTf32>(pr.side, side_off + static_cast<long long>(row) * pr.side_ld + col);
              float x = fmaf(P.gamma, a, P.beta * s);
              if (row == col) x += P.alpha;
              res = round_op<kTf32>(x);
              store_op<kTf32>(pr.out, out_off + idx, res);
              break;
            }
            case EPI_APPLY: {
              const float x = zero ? 0.f : (pr.first ? sc * a : a);
              res = round_op<kTf32>(x);
              store_op<kTf32>(pr.out, out_off + idx, res);
              break;
            }
            case EPI_APPLY_F32: {
              res = zero ? 0.f : (pr.first ? sc * a : a);
              reinterpret_cast<float*>(pr.out)[out_off + idx] = res;
              break;
            }
            default: {  // EPI_UPDATE: parameters are dense [M][N]
              const float u = zero ? 0.f : (pr.first ? sc * a : a);
              const long long pidx = static_cast<long long>(row) * pr.N + col;
              if (pr.param_dtype == MUON_BF16) {
                __nv_bfloat16* pp = reinterpret_cast<__nv_bfloat16*>(param_ptr);
                float p = __bfloat162float(pp[pidx]);
                if (pr.wd_factor != 1.f) p = bf16_round(p * pr.wd_factor);
                pp[pidx] = __float2bfloat16_rn(fmaf(-pr.eff, bf16_round(u), p));
              } else {
                float* pp = reinterpret_cast<float*>(param_ptr);
                float p = pp[pidx];
                if (pr.wd_factor != 1.f) p = p * pr.wd_factor;
                pp[pidx] = fmaf(-pr.eff, u, p);
              }
              res = u;
              break;
            }
          }
          buf[r * EPI_PITCH + lane] = res;
        }
        __syncwarp();
        if (pr.symmetric) {
          // Row mode: lane = row; store the strict upper part mirrored (coalesced).
          const int row = row0 + lane;
          if (row < pr.M) {
            for (int j = 0; j < 32; ++j) {
              const int c2 = col0 + j;
              if (c2 > row && c2 < pr.N)
                store_op<kTf32>(pr.out, out_off + static_cast<long long>(c2) * pr.out_ld + row,
                                buf[lane * EPI_PITCH + j]);
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// =====================================================================
// Host side: tensor maps, plan construction and launch.

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// A 3-D operand view [batch][outer][inner] with element strides ld (outer)
// and bs (batch). `box_outer` rows are loaded per TMA request, 128 bytes of
// the inner dimension each.
static int encode_operand(CUtensorMap* map, const void* base, int es, long long inner,
                          long long outer, long long batch, long long ld, long long bs,
                          int box_outer, bool mn_major = false) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return set_error(MUON_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return set_error(MUON_ERR_ARG, "NS operand buffer is not 16-byte aligned");
  if (((ld * es) & 15) != 0 || ((bs * es) & 15) != 0)
    return set_error(MUON_ERR_ARG, "NS operand leading dimension is not a multiple of 16 bytes");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * es), static_cast<cuuint64_t>(bs * es)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / es), static_cast<cuuint32_t>(box_outer), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  (mn_major && es == 4) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char msg[160];
    snprintf(msg, sizeof(msg), "cuTensorMapEncodeTiled failed (%d) for %lldx%lldx%lld ld=%lld", int(r),
             batch, outer, inner, ld);
    return set_error(MUON_ERR_CUDA, msg);
  }
  return MUON_OK;
}

}  // namespace muon

struct muon_ns_plan {
  int op_dtype;
  int steps;
  int n_classes;
  int num_sms;
  std::vector<muon::GemmParams> launches;  // 3 * steps
  std::vector<int> last_class_of_problem;  // final-apply launch: problem -> class
};

namespace muon {

static int tiles_per_matrix(int M, int N, bool symmetric, int* tm, int* tn) {
  *tm = (M + BM - 1) / BM;
  *tn = (N + BN - 1) / BN;
  if (!symmetric) return (*tm) * (*tn);
  int total = 0;
  for (int ti = 0; ti < *tm; ++ti) total += *tn - (ti >> 1);
  return total;
}

int64_t ns_class_workspace_bytes(int32_t rows, int32_t cols, int32_t count, int op_dtype) {
  if (rows <= 0 || cols <= 0 || count <= 0) return 0;
  const int es = op_dtype == MUON_BF16 ? 2 : 4;
  const int align_el = 16 / es;
  const int64_t m = std::min(rows, cols);
  const int64_t ld_x = (cols + align_el - 1) / align_el * align_el;
  const int64_t ld_m = (m + align_el - 1) / align_el * align_el;
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  return 2 * up(int64_t(count) * rows * ld_x * es) + 2 * up(int64_t(count) * m * ld_m * es);
}

int ns_class_layout(muon_ns_class* cls, void* base, int op_dtype) {
  if (!cls || !base) return set_error(MUON_ERR_ARG, "null class or workspace");
  if ((reinterpret_cast<uintptr_t>(base) & 255u) != 0)
    return set_error(MUON_ERR_ARG, "NS workspace must be 256-byte aligned");
  const int es = op_dtype == MUON_BF16 ? 2 : 4;
  const int align_el = 16 / es;
  const int64_t rows = cls->rows, cols = cls->cols, count = cls->count;
  const int64_t m = std::min(rows, cols);
  cls->ld_x = (cols + align_el - 1) / align_el * align_el;
  cls->ld_m = (m + align_el - 1) / align_el * align_el;
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  const int64_t xb = up(count * rows * cls->ld_x * es);
  const int64_t mb = up(count * m * cls->ld_m * es);
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  cls->x0 = p;
  cls->x1 = p + xb;
  cls->ap = p + 2 * xb;
  cls->mm = p + 2 * xb + mb;
  return MUON_OK;
}

int ns_plan_create(const muon_ns_class* classes, int n_classes, int op_dtype, int steps,
                   muon_ns_plan** plan_out) {
  if (!plan_out) return set_error(MUON_ERR_ARG, "plan_out is null");
  *plan_out = nullptr;
  if (op_dtype != MUON_TF32 && op_dtype != MUON_BF16)
    return set_error(MUON_ERR_ARG, "op_dtype must be MUON_TF32 or MUON_BF16");
  if (steps < 1) return set_error(MUON_ERR_UNSUPPORTED, "Newton-Schulz plans need steps >= 1");
  if (n_classes < 1 || n_classes > kMaxProblems)
    return set_error(MUON_ERR_ARG, "n_classes must be in [1, 16]");
  const int es = op_dtype == MUON_BF16 ? 2 : 4;
  for (int c = 0; c < n_classes; ++c) {
    const muon_ns_class& k = classes[c];
    if (k.rows <= 0 || k.cols <= 0 || k.count <= 0)
      return set_error(MUON_ERR_ARG, "class with an empty shape or count");
    if (!k.x0 || !k.x1 || !k.ap || !k.mm || !k.scales)
      return set_error(MUON_ERR_ARG, "class buffer pointer is null");
    if ((k.u_out == nullptr) == (k.params == nullptr))
      return set_error(MUON_ERR_ARG, "exactly one of u_out / params must be set per class");
    if (k.params && k.param_dtype != MUON_BF16 && k.param_dtype != MUON_F32)
      return set_error(MUON_ERR_ARG, "param_dtype must be MUON_BF16 or MUON_F32");
    const int m = std::min(k.rows, k.cols);
    if (k.ld_x < k.cols || k.ld_m < m) return set_error(MUON_ERR_ARG, "leading dimension too small");
    if (k.u_out && k.ld_u < k.cols) return set_error(MUON_ERR_ARG, "ld_u too small");
  }
  int dev = 0, sms = 0;
  if (check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return MUON_ERR_CUDA;
  if (check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count"))
    return MUON_ERR_CUDA;

  muon_ns_plan* plan = new muon_ns_plan();
  plan->op_dtype = op_dtype;
  plan->steps = steps;
  plan->n_classes = n_classes;
  plan->num_sms = sms;
  plan->launches.resize(3 * steps);

  const float alpha = float(kNsA + kNsB + kNsC);
  const float beta = float(kNsB + 2.0 * kNsC);
  const float gamma = float(kNsC);

  for (int it = 0; it < steps; ++it) {
    for (int phase = 0; phase < 3; ++phase) {
      GemmParams& L = plan->launches[3 * it + phase];
      memset(&L, 0, sizeof(L));
      L.alpha = alpha;
      L.beta = beta;
      L.gamma = gamma;
      // Order problems by K (largest first) so long tiles start early.
      std::vector<int> order(n_classes);
      for (int c = 0; c < n_classes; ++c) order[c] = c;
      auto kdim = [&](int c) {
        const muon_ns_class& k = classes[c];
        const int m = std::min(k.rows, k.cols), n = std::max(k.rows, k.cols);
        return phase == 0 ? n : m;
      };
      auto work = [&](int c) {
        const muon_ns_class& k = classes[c];
        const double m = std::min(k.rows, k.cols), n = std::max(k.rows, k.cols);
        return double(kdim(c)) * (phase == 2 ? m * n : m * m) * k.count;
      };
      std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
        if (kdim(x) != kdim(y)) return kdim(x) > kdim(y);
        return work(x) > work(y);
      });
      if (phase == 2 && it == steps - 1) plan->last_class_of_problem = order;
      int tile_begin = 0;
      for (int pi = 0; pi < n_classes; ++pi) {
        const int c = order[pi];
        const muon_ns_class& k = classes[c];
        GemmProblem& pr = L.prob[pi];
        const bool wide = k.rows <= k.cols;
        const int m = std::min(k.rows, k.cols), n = std::max(k.rows, k.cols);
        void* xin = (it % 2 == 0) ? k.x0 : k.x1;
        void* xout = (it % 2 == 0) ? k.x1 : k.x0;
        const long long xbs = static_cast<long long>(k.rows) * k.ld_x;
        const long long mbs = static_cast<long long>(m) * k.ld_m;
        int rc = MUON_OK;
        pr.batch = k.count;
        pr.scale = k.scales;
        if (phase == 0) {
          // A' = s^2 X X^T - I over the wide orientation.
          pr.M = m;
          pr.N = m;
          pr.K = n;
          pr.symmetric = 1;
          pr.epi = EPI_GRAM;
          pr.first = it == 0;
          pr.a_mn = pr.b_mn = wide ? 0 : 1;
          pr.out = k.ap;
          pr.out_ld = k.ld_m;
          pr.out_bs = mbs;
          if (wide) {
            rc = encode_operand(&L.map_a[pi], xin, es, k.cols, k.rows, k.count, k.ld_x, xbs, BM);
            if (!rc) rc = encode_operand(&L.map_b[pi], xin, es, k.cols, k.rows, k.count, k.ld_x, xbs, BN);
          } else {
            rc = encode_operand(&L.map_a[pi], xin, es, k.cols, k.rows, k.count, k.ld_x, xbs, 128 / es, true);
            if (!rc) rc = encode_operand(&L.map_b[pi], xin, es, k.cols, k.rows, k.count, k.ld_x, xbs, 128 / es, true);
          }
        } else if (phase == 1) {
          // M = alpha I + beta A' + gamma A'A' (A' symmetric: both operands K-major).
          pr.M = pr.N = pr.K = m;
          pr.symmetric = 1;
          pr.epi = EPI_POLY;
          pr.first = 0;
          pr.a_mn = pr.b_mn = 0;
          pr.out = k.mm;
          pr.out_ld = k.ld_m;
          pr.out_bs = mbs;
          pr.side = k.ap;
          pr.side_ld = k.ld_m;
          pr.side_bs = mbs;
          rc = encode_operand(&L.map_a[pi], k.ap, es, m, m, k.count, k.ld_m, mbs, BM);
          if (!rc) rc = encode_operand(&L.map_b[pi], k.ap, es, m, m, k.count, k.ld_m, mbs, BN);
        } else {
          // Wide: X' = M X (B operand MN-major). Tall: X' = X M (both K-major).
          pr.M = k.rows;
          pr.N = k.cols;
          pr.K = m;
          pr.symmetric = 0;
          pr.first = it == 0;
          const bool last = it == steps - 1;
          if (wide) {
            pr.a_mn = 0;
            pr.b_mn = 1;
            rc = encode_operand(&L.map_a[pi], k.mm, es, m, m, k.count, k.ld_m, mbs, BM);
            if (!rc) rc = encode_operand(&L.map_b[pi], xin, es, k.cols, k.rows, k.count, k.ld_x, xbs, 128 / es, true);
          } else {
            pr.a_mn = 0;
            pr.b_mn = 0;
            rc = encode_operand(&L.map_a[pi], xin, es, k.cols, k.rows, k.count, k.ld_x, xbs, BM);
            if (!rc) rc = encode_operand(&L.map_b[pi], k.mm, es, m, m, k.count, k.ld_m, mbs, BN);
          }
          if (!last) {
            pr.epi = EPI_APPLY;
            pr.out = xout;
            pr.out_ld = k.ld_x;
            pr.out_bs = xbs;
          } else if (k.u_out) {
            pr.epi = EPI_APPLY_F32;
            pr.out = k.u_out;
            pr.out_ld = k.ld_u;
            pr.out_bs = static_cast<long long>(k.rows) * k.ld_u;
          } else {
            pr.epi = EPI_UPDATE;
            pr.params = k.params;
            pr.param_dtype = k.param_dtype;
            pr.eff = 0.f;
            pr.wd_factor = 1.f;
          }
        }
        if (rc != MUON_OK) {
          delete plan;
          return rc;
        }
        pr.tiles_per_mat = tiles_per_matrix(pr.M, pr.N, pr.symmetric != 0, &pr.tiles_m, &pr.tiles_n);
        pr.tile_begin = tile_begin;
        tile_begin += pr.tiles_per_mat * pr.batch;
      }
      L.n_problems = n_classes;
      L.total_tiles = tile_begin;
    }
  }
  *plan_out = plan;
  return MUON_OK;
}

int ns_plan_run(const muon_ns_plan* plan, const float* eff, float wd_factor, int* err_dev,
                cudaStream_t stream) {
  if (!plan) return set_error(MUON_ERR_ARG, "plan is null");
  if (!err_dev) return set_error(MUON_ERR_ARG, "err_dev is null");
  static bool attr_set[2] = {false, false};
  const bool tf32 = plan->op_dtype == MUON_TF32;
  const void* fn = tf32 ? reinterpret_cast<const void*>(&ns_gemm_kernel<true>)
                        : reinterpret_cast<const void*>(&ns_gemm_kernel<false>);
  if (!attr_set[tf32]) {
    if (check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES),
                   "cudaFuncSetAttribute(ns_gemm)"))
      return MUON_ERR_CUDA;
    attr_set[tf32] = true;
  }
  const int n = static_cast<int>(plan->launches.size());
  for (int i = 0; i < n; ++i) {
    GemmParams L = plan->launches[i];
    L.err = err_dev;
    if (i == n - 1) {
      for (int pi = 0; pi < L.n_problems; ++pi) {
        if (L.prob[pi].epi == EPI_UPDATE) {
          if (!eff) return set_error(MUON_ERR_ARG, "eff is required for in-place parameter updates");
          L.prob[pi].eff = eff[plan->last_class_of_problem[pi]];
          L.prob[pi].wd_factor = wd_factor;
        }
      }
    }
    if (L.total_tiles == 0) continue;
    const int grid = std::min(L.total_tiles, plan->num_sms);
    if (tf32)
      ns_gemm_kernel<true><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(L);
    else
      ns_gemm_kernel<false><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(L);
    if (check_cuda(cudaGetLastError(), "ns_gemm launch")) return MUON_ERR_CUDA;
  }
  return MUON_OK;
}

void ns_plan_destroy(muon_ns_plan* plan) { delete plan; }

}  // namespace muon
