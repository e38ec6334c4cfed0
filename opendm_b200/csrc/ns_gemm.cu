// Grouped tcgen05/TMEM GEMMs for the Newton-Schulz orthogonalisation
// (reference: zeropower_via_newtonschulz5, opendm/optimizer/muon_adamw.py:101-128).
//
// One launch evaluates one phase of one Newton-Schulz iteration for every
// matrix of every shape class:
//   phase 0 (gram):  A' = s^2 X X^T - I and B' = gamma A' + beta I
//                                                     symmetric m x m, K = n
//   phase 1 (poly):  M  = alpha I + A' B'            symmetric m x m, K = m
//   phase 2 (apply): X  = s M X   (wide)  |  X = s X M  (tall: X kept as the
//                    parameter's n x m layout, which is the transpose)
// s is the per-matrix Frobenius scale on the first iteration and 1 after it
// (fp16 operands are stored pre-normalised and power-of-two scaled instead).
// The last apply writes the update U in fp32 or in the parameter dtype.
//
// Kernel structure: clusters of 2 CTAs (one per SM), persistent, static
// round-robin over 256 x 256 tiles. The pair issues cta_group::2 MMAs: CTA r
// holds rows [128 r, 128 r + 128) of the tile's A operand and of its B
// operand, and receives rows [128 r, 128 r + 128) of D in its own TMEM, so
// each SM loads half of B (32 KB per 64-deep K stage instead of 48 KB).
//   warp 0      TMA producer (both CTAs): a 6-stage ring; the bytes of both
//               CTAs complete on the leader CTA's full barrier
//   warp 1      TMEM allocation (both CTAs); single-thread MMA issuer (leader)
//   warps 2..5  epilogue (both CTAs): tcgen05.ld -> registers -> swizzled
//               shared-memory staging -> one TMA tensor store per 32 x 32
//               chunk; a symmetric C stores its upper 256 x 256 blocks only,
//               and a later product reads a block below the diagonal as
//               the MN-major transpose of the stored block
// Accumulators: two 128 x 256 fp32 buffers per CTA in TMEM (all 512 columns),
// so the epilogue of tile i overlaps the main loop of tile i+1. Each CTA
// loads its own operand halves with plain (single-destination) TMA loads.
// Operands are bf16 (kind::f16) or tf32 (kind::tf32); either way a stage
// holds 128 bytes of K per row, so the byte geometry is identical.

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace muon {

constexpr int BM = 128;          // rows of D per CTA
constexpr int PAIR_M = 2 * BM;   // rows of D per CTA pair (one tile)
constexpr int BN = 256;          // columns of D per tile
constexpr int BN_CTA = BN / 2;   // rows of the B operand each CTA of the pair holds
constexpr int STAGES = 6;
constexpr int A_STAGE_BYTES = BM * 128;
constexpr int B_STAGE_BYTES = BN_CTA * 128;
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int EPI_WARPS = 4;
constexpr int NUM_THREADS = 64 + EPI_WARPS * 32;
constexpr int EPI_WARP_BYTES = 8192;  // per epilogue warp: ring of TMA-store staging buffers
constexpr int EPI_BYTES = EPI_WARPS * EPI_WARP_BYTES;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
constexpr int TMEM_COLS = 2 * BN;
constexpr int kMaxProblems = 32;  // up to two problems per class per launch

enum EpiKind : int { EPI_GRAM = 0, EPI_POLY = 1, EPI_APPLY = 2, EPI_U_F32 = 3, EPI_U_BF16 = 4 };

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
  int a_sym, b_sym;  // operand is a symmetric m x m matrix stored as its upper 256 x 256 blocks
  int symmetric;   // output is symmetric: only its upper 256 x 256 blocks are computed and stored
  int epi;
  int first;       // apply the per-matrix input scale
  int split;       // operands stored as fp16 hi/lo pairs (batch slots 2g, 2g+1): K runs three times
  float mul;       // constant multiplier of the accumulator (power of two)
  float omul;      // poly: multiplier of the stored M / P (power of two)
  float omul3;     // gram: of the stored A; poly: of the stored Q (power of two)
  const void* out3;  // optional third output (gram: A; poly: Q); non-null when map_out3 is set
  const float* scale;
};

struct GemmParams {
  CUtensorMap map_a[kMaxProblems];
  CUtensorMap map_b[kMaxProblems];
  CUtensorMap map_out[kMaxProblems];   // D (A', M, X or U): 32 x 32 store boxes
  CUtensorMap map_out2[kMaxProblems];  // gram: B'
  CUtensorMap map_out3[kMaxProblems];  // gram: A; poly: Q (only where out3 is set)
  CUtensorMap map_at[kMaxProblems];    // a_sym: the A operand with MN-major boxes, for transposed blocks
  CUtensorMap map_bt[kMaxProblems];    // b_sym: the same for the B operand
  GemmProblem prob[kMaxProblems];
  int n_problems;
  int total_tiles;
  float alpha, beta, gamma;
  int* err;
};

// The whole launch descriptor is one __grid_constant__ kernel parameter.
static_assert(sizeof(GemmParams) <= 32764, "GemmParams exceeds the kernel parameter limit");

struct TileCoord {
  int p, g, ti, tj;
};

// Symmetric m x m operands keep only their 256 x 256 blocks on and above the
// diagonal. The K range [k0, k0 + stage) of operand rows in block `block`
// lies in a block below the diagonal when k0 / 256 < block; that stage reads
// the transposed block (k0 / 256, block) instead. Both CTAs of a pair hold
// rows of the same 256-row block, so they agree on every stage's layout.
__device__ __forceinline__ bool below_diagonal(int sym, int block, int k0) { return sym && k0 / PAIR_M < block; }

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
    // Square tiles: row block ti holds column blocks [ti, tiles_n), exactly
    // the tiles that contain an element with col >= row.
    int ti = 0;
    while (true) {
      const int cnt = pr.tiles_n - ti;
      if (lt < cnt) {
        c.tj = ti + lt;
        break;
      }
      lt -= cnt;
      ++ti;
    }
    c.ti = ti;
  }
  return c;
}

template <int kOp>
__device__ __forceinline__ void store_op(void* base, long long idx, float v) {
  if constexpr (kOp == kOpTf32) {
    reinterpret_cast<float*>(base)[idx] = v;
  } else if constexpr (kOp == kOpBf16) {
    reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v);
  }
}

template <int kOp>
__device__ __forceinline__ float round_op(float v) {
  if constexpr (kOp == kOpTf32) {
    return round_tf32(v);
  } else if constexpr (kOp == kOpBf16) {
    return bf16_round(v);
  } else {
    return f16_round(v);
  }
}

template <int kOp>
__device__ __forceinline__ float load_op(const void* base, long long idx) {
  if constexpr (kOp == kOpTf32) {
    return reinterpret_cast<const float*>(base)[idx];
  } else if constexpr (kOp == kOpBf16) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
  } else {
    return __half2float(reinterpret_cast<const __half*>(base)[idx]);
  }
}

// ------------------------------------------------------------ epilogue I/O
// A warp stores its 32 x 32 chunk of D through a ring of shared-memory
// buffers with one TMA store per chunk. The buffers use the layout of the
// output tensor map's swizzle (64B for 2-byte outputs, 128B for 4-byte ones),
// which also makes the 16-byte shared stores below bank-conflict free.

// Row-major staging: lane = row, `w` holds the row packed (2-byte: 16 words).
__device__ __forceinline__ void stage_rows_16(uint8_t* buf, int lane, const uint32_t (&w)[16]) {
  const uint32_t base = smem_u32(buf) + lane * 64;
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    st_shared_v4(base + ((k ^ sw) << 4), w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
}

__device__ __forceinline__ void stage_rows_32(uint8_t* buf, int lane, const uint32_t (&w)[32]) {
  const uint32_t base = smem_u32(buf) + lane * 128;
  const int sw = lane & 7;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    st_shared_v4(base + ((k ^ sw) << 4), w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
}

// Rounds 32 fp32 values of one row into output words.
// kind: 0 = fp32 (raw), 1 = tf32 (rna), 2 = fp16, 3 = bf16.
template <int kWords>
__device__ __forceinline__ void pack_row(const float (&x)[32], int kind, uint32_t (&w)[kWords]) {
  if constexpr (kWords == 32) {
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(kind == 1 ? round_tf32(x[i]) : x[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (kind == 2) {
        const __half2 h = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
  }
}

// Per-warp ring of staging buffers: 4 x 2 KB (2-byte outputs) or 2 x 4 KB.
struct StoreRing {
  uint8_t* base;
  int issued;
  int out_bytes;
};

template <int kOutBytes>
__device__ __forceinline__ uint8_t* ring_acquire(StoreRing& ring, int lane) {
  constexpr int kBuf = kOutBytes == 2 ? 2048 : 4096;
  constexpr int kN = EPI_WARP_BYTES / kBuf;
  if (ring.out_bytes != kOutBytes) {  // buffer size changes: let every store finish reading
    if (lane == 0) bulk_wait_group_read<0>();
    __syncwarp();
    ring.issued = 0;
    ring.out_bytes = kOutBytes;
  } else if (ring.issued >= kN) {
    if (lane == 0) bulk_wait_group_read<kN - 1>();  // the store that used this buffer is done
    __syncwarp();
  }
  return ring.base + (ring.issued % kN) * kBuf;
}

__device__ __forceinline__ void ring_store(StoreRing& ring, uint8_t* buf, const CUtensorMap* map, int lane, int x,
                                           int y, int z) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_3d(map, buf, x, y, z);
    bulk_commit_group();
  }
  ++ring.issued;
}

// Store one chunk (row-major words of this lane's row) at (x = col0, y = row0).
template <int kWords>
__device__ __forceinline__ void store_chunk(StoreRing& ring, const CUtensorMap* map, int lane, const uint32_t (&w)[kWords],
                                            int col0, int row0, int g) {
  constexpr int kOutBytes = kWords == 32 ? 4 : 2;
  uint8_t* buf = ring_acquire<kOutBytes>(ring, lane);
  if constexpr (kWords == 32) stage_rows_32(buf, lane, w); else stage_rows_16(buf, lane, w);
  ring_store(ring, buf, map, lane, col0, row0, g);
}

// Store one chunk of a Newton-Schulz operand output (32 fp32 values of this
// lane's row), rounded to the operand type. With split operands the value
// goes out as a pair: hi = round(x) at batch slot 2g and lo = round(x - hi)
// at 2g + 1 (x - hi is exact in fp32), so hi + lo carries ~22 bits.
template <int kOp, int kWords>
__device__ __forceinline__ void store_operand(StoreRing& ring, const CUtensorMap* map, int lane, const float (&x)[32],
                                              int kind, int col0, int row0, int g, bool split) {
  uint32_t w[kWords];
  pack_row<kWords>(x, kind, w);
  store_chunk<kWords>(ring, map, lane, w, col0, row0, split ? 2 * g : g);
  if (split) {
    float lo[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) lo[i] = x[i] - round_op<kOp>(x[i]);
    pack_row<kWords>(lo, kind, w);
    store_chunk<kWords>(ring, map, lane, w, col0, row0, 2 * g + 1);
  }
}

template <int kOp>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    ns_gemm_kernel(const __grid_constant__ GemmParams P) {
  constexpr bool kTf32 = kOp == kOpTf32;
  constexpr int ES = kTf32 ? 4 : 2;
  constexpr int BKE = 128 / ES;     // K elements per stage == MN elements per swizzle atom
  constexpr int UMMA_K = 32 / ES;   // K elements per tcgen05.mma
  constexpr int KSTEPS = BKE / UMMA_K;
  // MN-major operands: 16-bit types use the 128B swizzle (8-row K groups, SBO 1024);
  // tf32 must use the 32-byte-atom 128B swizzle (4-row K groups, SBO 512).
  constexpr uint32_t kMnLayout = kTf32 ? kLayoutSw128Base32 : kLayoutSw128;
  constexpr uint32_t kMnSbo = kTf32 ? 512 : 1024;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stage_a = smem;
  uint8_t* stage_b = smem + STAGES * A_STAGE_BYTES;
  uint8_t* epi_buf = smem + STAGES * STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES + EPI_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: leader (issues the MMAs)
  const int cluster_id = blockIdx.x >> 1;
  const int n_clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS);  // epilogue warps of both CTAs (leader's copy is used)
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
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // peer barriers initialised and TMEM allocated in both CTAs
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
      for (int t = cluster_id; ok && t < P.total_tiles; t += n_clusters) {
        const TileCoord tc = decode_tile(P, t);
        const GemmProblem& pr = P.prob[tc.p];
        const int kb_count = (pr.K + BKE - 1) / BKE;
        const int kb_total = pr.split ? 3 * kb_count : kb_count;
        const int m0 = tc.ti * PAIR_M + static_cast<int>(rank) * BM;
        const int n0 = tc.tj * BN + static_cast<int>(rank) * BN_CTA;
        for (int kbi = 0; kbi < kb_total; ++kbi) {
          // Split operands: K segment 0 = hi * hi, 1 = hi * lo, 2 = lo * hi.
          const int seg = pr.split ? kbi / kb_count : 0;
          const int kb = kbi - seg * kb_count;
          const int za = pr.split ? 2 * tc.g + (seg == 2 ? 1 : 0) : tc.g;
          const int zb = pr.split ? 2 * tc.g + (seg == 1 ? 1 : 0) : tc.g;
          if (!mbar_wait(&empty[stage], phase ^ 1u, P.err, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
          const uint32_t bar = map_shared_rank(smem_u32(&full[stage]), 0);
          uint8_t* sa = stage_a + stage * A_STAGE_BYTES;
          uint8_t* sb = stage_b + stage * B_STAGE_BYTES;
          const int k0 = kb * BKE;
          // A block of a symmetric operand below its diagonal is read from the
          // stored block above it, as an MN-major tile (the MMA issuer makes the
          // same choice for the stage's descriptors).
          const bool a_t = below_diagonal(pr.a_sym, tc.ti, k0);
          const bool b_t = below_diagonal(pr.b_sym, tc.tj, k0);
          const CUtensorMap* map_a = a_t ? &P.map_at[tc.p] : &P.map_a[tc.p];
          const CUtensorMap* map_b = b_t ? &P.map_bt[tc.p] : &P.map_b[tc.p];
          if (!pr.a_mn && !a_t) {
            tma_load_3d_pair(sa, map_a, bar, k0, m0, za);
          } else {
#pragma unroll
            for (int j = 0; j < BM / BKE; ++j) tma_load_3d_pair(sa + j * BKE * 128, map_a, bar, m0 + j * BKE, k0, za);
          }
          if (!pr.b_mn && !b_t) {
            tma_load_3d_pair(sb, map_b, bar, k0, n0, zb);
          } else {
#pragma unroll
            for (int j = 0; j < BN_CTA / BKE; ++j)
              tma_load_3d_pair(sb + j * BKE * 128, map_b, bar, n0 + j * BKE, k0, zb);
          }
          issued[stage] = 1;
          issued_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: a stage is released (empty) only after the MMAs that read it
      // completed, which implies its loads landed.
      for (int s = 0; s < STAGES; ++s)
        if (issued[s]) mbar_wait(&empty[s], issued_phase[s], P.err, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    // ------------------------------------------------- MMA issuer (leader)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local_t = 0;
      bool ok = true;
      for (int t = cluster_id; ok && t < P.total_tiles; t += n_clusters, ++local_t) {
        const TileCoord tc = decode_tile(P, t);
        const GemmProblem& pr = P.prob[tc.p];
        const int kb_single = (pr.K + BKE - 1) / BKE;
        const int kb_count = kb_single * (pr.split ? 3 : 1);
        const int acc = local_t & 1;
        const uint32_t acc_phase = (local_t >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, P.err, kDevTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0, kin = 0; kb < kb_count; ++kb, kin = (kin + 1 == kb_single) ? 0 : kin + 1) {
          if (!mbar_wait(&full[stage], phase, P.err, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // the stage's operand layouts, as the producer loaded them
          const bool a_mn = pr.a_mn || below_diagonal(pr.a_sym, tc.ti, kin * BKE);
          const bool b_mn = pr.b_mn || below_diagonal(pr.b_sym, tc.tj, kin * BKE);
          const uint32_t idesc = make_idesc(kOp, PAIR_M, BN, a_mn, b_mn);
          const uint32_t a_addr = smem_u32(stage_a + stage * A_STAGE_BYTES);
          const uint32_t b_addr = smem_u32(stage_b + stage * B_STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < KSTEPS; ++kk) {
            const uint64_t ad = a_mn ? make_sw128_desc(a_addr + kk * UMMA_K * 128, BKE * 128, kMnSbo, kMnLayout)
                                     : make_sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = b_mn ? make_sw128_desc(b_addr + kk * UMMA_K * 128, BKE * 128, kMnSbo, kMnLayout)
                                     : make_sw128_desc(b_addr + kk * 32, 16, 1024);
            umma_pair<kOp>(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          // Release the stage in both CTAs once these MMAs have read it.
          umma_commit_pair(smem_u32(&empty[stage]));
          umma_commit_pair(map_shared_rank(smem_u32(&empty[stage]), 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&tfull[acc]));
        umma_commit_pair(map_shared_rank(smem_u32(&tfull[acc]), 1));
      }
      // Drain: all issued MMAs complete before TMEM is released.
      umma_commit_pair(smem_u32(drain));
      mbar_wait(drain, 0, P.err, kDevTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    StoreRing ring{epi_buf + (warp - 2) * EPI_WARP_BYTES, 0, 0};
    const uint32_t leader_tempty0 = map_shared_rank(smem_u32(&tempty[0]), 0);
    const uint32_t leader_tempty1 = map_shared_rank(smem_u32(&tempty[1]), 0);
    // Output word kinds: 0 fp32, 1 tf32, 2 fp16, 3 bf16.
    constexpr int kOpKind = kOp == kOpTf32 ? 1 : kOp == kOpF16 ? 2 : 3;
    constexpr int kOpWords = kOp == kOpTf32 ? 32 : 16;
    int local_t = 0;
    for (int t = cluster_id; t < P.total_tiles; t += n_clusters, ++local_t) {
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
      const float mul = pr.mul;
      const int row0 = tc.ti * PAIR_M + static_cast<int>(rank) * BM + quad * 32;
      const float f = pr.first ? sc * sc * mul : mul;  // gram: s^2 * mul
      const float fa = pr.first ? sc * mul : mul;      // apply: s * mul
      const int myrow = row0 + lane;
      const CUtensorMap* map1 = &P.map_out[tc.p];
      const CUtensorMap* map2 = &P.map_out2[tc.p];
      const CUtensorMap* map3 = &P.map_out3[tc.p];
      const bool has3 = pr.out3 != nullptr;

      for (int ch = 0; ch < BN / 32; ++ch) {
        const int col0 = tc.tj * BN + ch * 32;
        float v[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN + ch * 32, v);
        // Symmetric outputs: the tile table holds the blocks on and above the
        // diagonal only, each stored whole; consumers read the blocks below
        // the diagonal transposed from them (below_diagonal).
        if (row0 >= pr.M || col0 >= pr.N) continue;
        float x[32];
        const bool split = pr.split != 0;
        if (pr.epi == EPI_GRAM) {
          if (has3) {  // A itself, scaled for storage
            const float m3 = pr.omul3;
#pragma unroll
            for (int i = 0; i < 32; ++i) x[i] = zero ? 0.f : (v[i] * f) * m3;
            store_operand<kOp, kOpWords>(ring, map3, lane, x, kOpKind, col0, row0, tc.g, split);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float a = zero ? 0.f : v[i] * f;
            x[i] = (myrow == col0 + i) ? a - 1.f : a;  // A'
          }
          store_operand<kOp, kOpWords>(ring, map1, lane, x, kOpKind, col0, row0, tc.g, split);
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = fmaf(P.gamma, x[i], (myrow == col0 + i) ? P.beta : 0.f);  // B'
          store_operand<kOp, kOpWords>(ring, map2, lane, x, kOpKind, col0, row0, tc.g, split);
        } else if (pr.epi == EPI_POLY) {
          const float pm = pr.mul, om = pr.omul;
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = (myrow == col0 + i) ? fmaf(v[i], pm, P.alpha) : v[i] * pm;
          if (has3) {  // the same polynomial, stored a second time at another scale
            float y[32];
            const float m3 = pr.omul3;
#pragma unroll
            for (int i = 0; i < 32; ++i) y[i] = x[i] * m3;
            store_operand<kOp, kOpWords>(ring, map3, lane, y, kOpKind, col0, row0, tc.g, split);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] *= om;
          store_operand<kOp, kOpWords>(ring, map1, lane, x, kOpKind, col0, row0, tc.g, split);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = zero ? 0.f : v[i] * fa;
          if (pr.epi == EPI_APPLY) {
            store_operand<kOp, kOpWords>(ring, map1, lane, x, kOpKind, col0, row0, tc.g, split);
          } else if (pr.epi == EPI_U_BF16) {
            uint32_t w[16];
            pack_row<16>(x, 3, w);
            store_chunk<16>(ring, map1, lane, w, col0, row0, tc.g);
          } else {
            uint32_t w[32];
            pack_row<32>(x, 0, w);
            store_chunk<32>(ring, map1, lane, w, col0, row0, tc.g);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
    }
    if (lane == 0) bulk_wait_group_all();  // every TMA store of this warp has completed
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs done with TMEM and with each other's barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
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
static int op_bytes(int op) { return op == MUON_TF32 ? 4 : 2; }
// Split operands (MUON_F16X3) take two batch slots per matrix: hi, then lo.
static int op_halves(int op) { return op == MUON_F16X3 ? 2 : 1; }
static bool op_is_f16(int op) { return op == MUON_F16 || op == MUON_F16X3; }

static int encode_operand(CUtensorMap* map, const void* base, int op, long long inner,
                          long long outer, long long batch, long long ld, long long bs,
                          int box_outer, bool mn_major = false) {
  const int es = op_bytes(op);
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return set_error(MUON_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return set_error(MUON_ERR_ARG, "NS operand buffer is not 16-byte aligned");
  if (((ld * es) & 15) != 0 || ((bs * es) & 15) != 0)
    return set_error(MUON_ERR_ARG, "NS operand leading dimension is not a multiple of 16 bytes");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                        static_cast<cuuint64_t>(batch * op_halves(op))};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * es), static_cast<cuuint64_t>(bs * es)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / es), static_cast<cuuint32_t>(box_outer), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = op == MUON_TF32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : op == MUON_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 3,
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
  int sm_limit = 0;  // 0: every SM; else at most this many SMs per launch
  std::vector<muon::GemmParams> launches;  // non-empty launch slots, in order
};

namespace muon {

// Power-of-two scale S_it of the stored Newton-Schulz operand X at iteration
// `it` in fp16 mode, chosen so the entries have magnitude about 1: the input
// X0 has unit Frobenius norm (entries ~ 1/sqrt(rows*cols)), later iterates
// have singular values ~1 (entries ~ 1/sqrt(max(rows, cols))). Powers of two
// keep every rescaling exact. Other modes store X unscaled (1.0).
float ns_operand_scale(int32_t rows, int32_t cols, int iteration, int op_dtype) {
  if (!op_is_f16(op_dtype) || rows <= 0 || cols <= 0) return 1.0f;
  const double target = iteration == 0 ? std::sqrt(double(rows) * double(cols))
                                        : std::sqrt(double(std::max(rows, cols)));
  return std::ldexp(1.0f, static_cast<int>(std::lround(std::log2(target))));
}

static int tiles_per_matrix(int M, int N, bool symmetric, int* tm, int* tn) {
  *tm = (M + PAIR_M - 1) / PAIR_M;
  *tn = (N + BN - 1) / BN;
  if (!symmetric) return (*tm) * (*tn);
  int total = 0;
  for (int ti = 0; ti < *tm; ++ti) total += *tn - ti;  // square tiles: tj in [ti, tn)
  return total;
}

// Output view [batch][outer][inner] of element type `dtype` (MUON_*) for
// 32 x 32 TMA stores, swizzled like the epilogue's staging buffers.
static int encode_output(CUtensorMap* map, const void* base, int dtype, long long inner, long long outer,
                         long long batch, long long ld, long long bs) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return set_error(MUON_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int es = (dtype == MUON_F32 || dtype == MUON_TF32) ? 4 : 2;
  batch *= op_halves(dtype);  // split operand outputs: hi and lo slots
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return set_error(MUON_ERR_ARG, "NS output buffer is not 16-byte aligned");
  if (((ld * es) & 15) != 0 || ((bs * es) & 15) != 0)
    return set_error(MUON_ERR_ARG, "NS output leading dimension is not a multiple of 16 bytes");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * es), static_cast<cuuint64_t>(bs * es)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = es == 4             ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : op_is_f16(dtype) ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                     : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  es == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char msg[160];
    snprintf(msg, sizeof(msg), "cuTensorMapEncodeTiled (output) failed (%d) for %lldx%lldx%lld ld=%lld", int(r),
             batch, outer, inner, ld);
    return set_error(MUON_ERR_CUDA, msg);
  }
  return MUON_OK;
}

// ------------------------------------------------------------ algorithms
// MUON_NS_STANDARD runs every iteration on X (gram, poly, apply: 3 launches
// per iteration). MUON_NS_GRAM runs the iteration on the m x m gram matrix
// instead, for matrices with n noticeably larger than m:
//   X_k = P_{k-1} ... P_0 X_0 with P_j = a + b A_j + c A_j^2 (a polynomial of
//   A_j) and A_{j+1} = P_j A_j P_j = P_j (P_j A_j), since P_j and A_j commute.
// The product Q = P_j ... P_s is accumulated in m x m and applied to X only
// at the end of a segment of kGramSegment iterations, after which the gram
// matrix is recomputed from the new X (a restart: without it, rounding in the
// m x m products grows in the directions of small singular values). Per
// segment of L iterations: one gram (m^2 n), 4L - 3 symmetric m x m products
// and one apply (2 m^2 n), against L (3 m^2 n + m^3) for the standard form.
// Each launch slot of an iteration still holds three dependent phases, so
// both algorithms share launches; a segment end adds one apply launch.
constexpr int kGramSegment = 3;
constexpr int kGramMaxM = 32768;  // keeps the scaled fp16 values of A, P and Q finite

static double p2_near(double x) { return std::ldexp(1.0, static_cast<int>(std::lround(std::log2(x)))); }

// fp16 storage scales of the gram-form m x m matrices (1 for tf32): A, P, PA
// have eigenvalues below 3.5 and are stored times m/4; Q (a product of up to
// three P) below 41, stored times m/64.
static float gram_scale_a(int m, int op) { return op_is_f16(op) ? float(p2_near(m / 4.0)) : 1.0f; }
static float gram_scale_q(int m, int op) { return op_is_f16(op) ? float(p2_near(m / 64.0)) : 1.0f; }

int ns_gram_segment(int op_dtype) { return op_is_f16(op_dtype) || op_dtype == MUON_TF32 ? kGramSegment : 0; }

static double exec_flops(int rows, int cols, int steps, int algo) {
  const double m = std::min(rows, cols), n = std::max(rows, cols);
  auto kp = [](double k) { return std::ceil(k / 64.0) * 64.0; };
  const double t = std::ceil(m / 256.0);
  const double tile = 256.0 * 256.0 * 2.0;
  const double gram = t * (t + 1) / 2 * tile * kp(n);
  const double sq = t * (t + 1) / 2 * tile * kp(m);
  const double app = std::ceil(rows / 256.0) * std::ceil(cols / 256.0) * tile * kp(m);
  if (algo == MUON_NS_STANDARD) return steps * (gram + sq + app);
  double f = 0;
  for (int s0 = 0; s0 < steps; s0 += kGramSegment) {
    const int len = std::min(kGramSegment, steps - s0);
    f += gram + (4 * len - 3) * sq + app;
  }
  return f;
}

int ns_choose_algo(int32_t rows, int32_t cols, int op_dtype, int steps) {
  if (!op_is_f16(op_dtype) && op_dtype != MUON_TF32) return MUON_NS_STANDARD;
  if (rows <= 0 || cols <= 0 || steps < kGramSegment) return MUON_NS_STANDARD;
  if (std::min(rows, cols) > kGramMaxM) return MUON_NS_STANDARD;
  return exec_flops(rows, cols, steps, MUON_NS_GRAM) < 0.9 * exec_flops(rows, cols, steps, MUON_NS_STANDARD)
             ? MUON_NS_GRAM
             : MUON_NS_STANDARD;
}

int64_t ns_class_workspace_bytes(int32_t rows, int32_t cols, int32_t count, int op_dtype, int algo) {
  if (rows <= 0 || cols <= 0 || count <= 0) return 0;
  if (op_dtype != MUON_TF32 && op_dtype != MUON_BF16 && !op_is_f16(op_dtype)) return 0;
  if (algo != MUON_NS_STANDARD && algo != MUON_NS_GRAM) return 0;
  const int es = op_bytes(op_dtype);
  const int align_el = 16 / es;
  const int64_t m = std::min(rows, cols);
  const int64_t ld_x = (cols + align_el - 1) / align_el * align_el;
  const int64_t ld_m = (m + align_el - 1) / align_el * align_el;
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  const int n_mm = algo == MUON_NS_GRAM ? 7 : 3;
  const int64_t h = op_halves(op_dtype);
  return 2 * up(h * count * rows * ld_x * es) + n_mm * up(h * count * m * ld_m * es);
}

int ns_class_layout(muon_ns_class* cls, void* base, int op_dtype) {
  if (!cls || !base) return set_error(MUON_ERR_ARG, "null class or workspace");
  if ((reinterpret_cast<uintptr_t>(base) & 255u) != 0)
    return set_error(MUON_ERR_ARG, "NS workspace must be 256-byte aligned");
  if (op_dtype != MUON_TF32 && op_dtype != MUON_BF16 && !op_is_f16(op_dtype))
    return set_error(MUON_ERR_ARG, "op_dtype must be MUON_TF32, MUON_BF16, MUON_F16 or MUON_F16X3");
  if (cls->algo != MUON_NS_STANDARD && cls->algo != MUON_NS_GRAM)
    return set_error(MUON_ERR_ARG, "algo must be MUON_NS_STANDARD or MUON_NS_GRAM");
  const int es = op_bytes(op_dtype);
  const int align_el = 16 / es;
  const int64_t rows = cls->rows, cols = cls->cols, count = cls->count;
  const int64_t m = std::min(rows, cols);
  cls->ld_x = (cols + align_el - 1) / align_el * align_el;
  cls->ld_m = (m + align_el - 1) / align_el * align_el;
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  const int64_t h = op_halves(op_dtype);
  const int64_t xb = up(h * count * rows * cls->ld_x * es);
  const int64_t mb = up(h * count * m * cls->ld_m * es);
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  cls->x0 = p;
  cls->x1 = p + xb;
  cls->ap = p + 2 * xb;
  cls->bp = p + 2 * xb + mb;
  cls->mm = p + 2 * xb + 2 * mb;
  if (cls->algo == MUON_NS_GRAM) {
    cls->aa = p + 2 * xb + 3 * mb;
    cls->pa = p + 2 * xb + 4 * mb;
    cls->qa = p + 2 * xb + 5 * mb;
    cls->qb = p + 2 * xb + 6 * mb;
  } else {
    cls->aa = cls->pa = cls->qa = cls->qb = nullptr;
  }
  return MUON_OK;
}

namespace {

struct OpDesc {
  const void* base = nullptr;
  long long inner = 0, outer = 0, ld = 0, bs = 0;
  int box = 0;
  bool mn = false;
  bool sym = false;  // a symmetric m x m buffer holding its upper 256 x 256 blocks
};

struct OutDesc {
  const void* base = nullptr;
  int dtype = 0;
  long long inner = 0, outer = 0, ld = 0, bs = 0;
};

// One GEMM problem of a launch before its tensor maps are encoded.
struct Pending {
  GemmProblem pr;
  OpDesc a, b;
  OutDesc o1, o2, o3;
  double work = 0;
};

struct ClassGeom {
  const muon_ns_class* k;
  int op, es, m, n;
  bool wide;
  long long xbs, mbs;

  // m x m operands are symmetric and stored as their upper 256 x 256 blocks
  OpDesc mat(const void* buf, int box) const { return OpDesc{buf, m, m, k->ld_m, mbs, box, false, true}; }
  OutDesc mat_out(const void* buf) const { return OutDesc{buf, op, m, m, k->ld_m, mbs}; }
  OutDesc x_out(const void* buf) const { return OutDesc{buf, op, k->cols, k->rows, k->ld_x, xbs}; }
  OutDesc u_out() const {
    return OutDesc{k->u_out, k->u_dtype, k->cols, k->rows, k->ld_u, static_cast<long long>(k->rows) * k->ld_u};
  }

  Pending base(int M, int N, int K, int sym, int epi) const {
    Pending p;
    memset(&p.pr, 0, sizeof(p.pr));
    p.pr.M = M;
    p.pr.N = N;
    p.pr.K = K;
    p.pr.batch = k->count;
    p.pr.symmetric = sym;
    p.pr.epi = epi;
    p.pr.mul = 1.0f;
    p.pr.omul = 1.0f;
    p.pr.omul3 = 1.0f;
    p.pr.scale = k->scales;
    p.pr.split = op == MUON_F16X3 ? 1 : 0;
    p.work = double(M) * N * K * k->count * (p.pr.split ? 3 : 1);
    return p;
  }

  // A' = f X X^T - I and B' (and A * a_scale when `a_out`), K = n.
  Pending gram_x(const void* xin, bool first, float mul, void* a_out, float a_scale) const {
    Pending p = base(m, m, n, 1, EPI_GRAM);
    p.pr.first = first;
    p.pr.mul = mul;
    p.pr.a_mn = p.pr.b_mn = wide ? 0 : 1;
    if (wide) {
      p.a = OpDesc{xin, k->cols, k->rows, k->ld_x, xbs, BM, false};
      p.b = OpDesc{xin, k->cols, k->rows, k->ld_x, xbs, BN_CTA, false};
    } else {
      p.a = OpDesc{xin, k->cols, k->rows, k->ld_x, xbs, 128 / es, true};
      p.b = OpDesc{xin, k->cols, k->rows, k->ld_x, xbs, 128 / es, true};
    }
    p.o1 = mat_out(k->ap);
    p.o2 = mat_out(k->bp);
    if (a_out) {
      p.o3 = mat_out(a_out);
      p.pr.omul3 = a_scale;
    }
    return p;
  }

  // Symmetric product of two symmetric m x m operands (both K-major) into
  // the m x m buffer `out`.
  Pending sym(const void* lhs, const void* rhs, int epi, float mul, const void* out) const {
    Pending p = base(m, m, m, 1, epi);
    p.pr.mul = mul;
    p.a = mat(lhs, BM);
    p.b = mat(rhs, BN_CTA);
    p.o1 = mat_out(out);
    return p;
  }

  // X' = M X (wide) or X M (tall) with M symmetric m x m; writes X' (op
  // dtype) or, when `xout` is null, U.
  Pending apply(const void* mbuf, const void* xin, bool first, float mul, const void* xout) const {
    Pending p = base(k->rows, k->cols, m, 0, xout ? EPI_APPLY : (k->u_dtype == MUON_BF16 ? EPI_U_BF16 : EPI_U_F32));
    p.pr.first = first;
    p.pr.mul = mul;
    if (wide) {
      p.pr.a_mn = 0;
      p.pr.b_mn = 1;
      p.a = mat(mbuf, BM);
      p.b = OpDesc{xin, k->cols, k->rows, k->ld_x, xbs, 128 / es, true};
    } else {
      p.pr.a_mn = 0;
      p.pr.b_mn = 0;
      p.a = OpDesc{xin, k->cols, k->rows, k->ld_x, xbs, BM, false};
      p.b = mat(mbuf, BN_CTA);
    }
    p.o1 = xout ? x_out(xout) : u_out();
    return p;
  }
};

int encode_pending(GemmParams& L, int pi, const Pending& q, int op) {
  const int mn_box = 128 / op_bytes(op);  // MN-major boxes: one stage of K by one swizzle atom of M
  int rc = encode_operand(&L.map_a[pi], q.a.base, op, q.a.inner, q.a.outer, q.pr.batch, q.a.ld, q.a.bs, q.a.box,
                          q.a.mn);
  if (!rc)
    rc = encode_operand(&L.map_b[pi], q.b.base, op, q.b.inner, q.b.outer, q.pr.batch, q.b.ld, q.b.bs, q.b.box,
                        q.b.mn);
  if (!rc && q.a.sym)
    rc = encode_operand(&L.map_at[pi], q.a.base, op, q.a.inner, q.a.outer, q.pr.batch, q.a.ld, q.a.bs, mn_box, true);
  if (!rc && q.b.sym)
    rc = encode_operand(&L.map_bt[pi], q.b.base, op, q.b.inner, q.b.outer, q.pr.batch, q.b.ld, q.b.bs, mn_box, true);
  if (!rc)
    rc = encode_output(&L.map_out[pi], q.o1.base, q.o1.dtype, q.o1.inner, q.o1.outer, q.pr.batch, q.o1.ld,
                       q.o1.bs);
  if (!rc && q.o2.base)
    rc = encode_output(&L.map_out2[pi], q.o2.base, q.o2.dtype, q.o2.inner, q.o2.outer, q.pr.batch, q.o2.ld,
                       q.o2.bs);
  if (!rc && q.o3.base)
    rc = encode_output(&L.map_out3[pi], q.o3.base, q.o3.dtype, q.o3.inner, q.o3.outer, q.pr.batch, q.o3.ld,
                       q.o3.bs);
  if (rc) return rc;
  GemmProblem& pr = L.prob[pi];
  pr = q.pr;
  pr.a_sym = q.a.sym ? 1 : 0;
  pr.b_sym = q.b.sym ? 1 : 0;
  pr.out3 = q.o3.base;
  return MUON_OK;
}

}  // namespace

int ns_plan_create(const muon_ns_class* classes, int n_classes, int op_dtype, int steps,
                   muon_ns_plan** plan_out) {
  if (!plan_out) return set_error(MUON_ERR_ARG, "plan_out is null");
  *plan_out = nullptr;
  if (op_dtype != MUON_TF32 && op_dtype != MUON_BF16 && !op_is_f16(op_dtype))
    return set_error(MUON_ERR_ARG, "op_dtype must be MUON_TF32, MUON_BF16, MUON_F16 or MUON_F16X3");
  if (steps < 1) return set_error(MUON_ERR_UNSUPPORTED, "Newton-Schulz plans need steps >= 1");
  if (n_classes < 1 || n_classes > kMaxProblems / 2)
    return set_error(MUON_ERR_ARG, "n_classes must be in [1, 16]");
  bool any_gram = false;
  for (int c = 0; c < n_classes; ++c) {
    const muon_ns_class& k = classes[c];
    if (k.rows <= 0 || k.cols <= 0 || k.count <= 0)
      return set_error(MUON_ERR_ARG, "class with an empty shape or count");
    if (!k.x0 || !k.x1 || !k.ap || !k.bp || !k.mm || !k.scales || !k.u_out)
      return set_error(MUON_ERR_ARG, "class buffer pointer is null");
    if (k.u_dtype != MUON_BF16 && k.u_dtype != MUON_F32)
      return set_error(MUON_ERR_ARG, "u_dtype must be MUON_BF16 or MUON_F32");
    const int m = std::min(k.rows, k.cols);
    if (k.ld_x < k.cols || k.ld_m < m) return set_error(MUON_ERR_ARG, "leading dimension too small");
    if (k.ld_u < k.cols) return set_error(MUON_ERR_ARG, "ld_u too small");
    if (k.algo == MUON_NS_GRAM) {
      if (op_dtype == MUON_BF16)
        return set_error(MUON_ERR_UNSUPPORTED, "MUON_NS_GRAM needs MUON_F16, MUON_F16X3 or MUON_TF32");
      if (m > kGramMaxM) return set_error(MUON_ERR_UNSUPPORTED, "MUON_NS_GRAM supports min(rows, cols) <= 32768");
      if (!k.aa || !k.pa || !k.qa || !k.qb) return set_error(MUON_ERR_ARG, "gram class buffer pointer is null");
      any_gram = true;
    } else if (k.algo != MUON_NS_STANDARD) {
      return set_error(MUON_ERR_ARG, "algo must be MUON_NS_STANDARD or MUON_NS_GRAM");
    }
    if ((k.flags & ~MUON_NS_INPUT_SCALED) != 0) return set_error(MUON_ERR_ARG, "unknown muon_ns_class flags");
  }
  int dev = 0, sms = 0;
  if (check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return MUON_ERR_CUDA;
  if (check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count"))
    return MUON_ERR_CUDA;

  const bool f16 = op_is_f16(op_dtype);
  const int es = op_bytes(op_dtype);

  // Launch slots: three phases per iteration, plus one apply slot at the end
  // of each gram segment when a class uses the gram form.
  std::vector<int> slot_of(3 * steps), ex_slot(steps, -1);
  int n_slots = 0;
  for (int it = 0; it < steps; ++it) {
    for (int ph = 0; ph < 3; ++ph) slot_of[3 * it + ph] = n_slots++;
    if (any_gram && (it % kGramSegment == kGramSegment - 1 || it == steps - 1)) ex_slot[it] = n_slots++;
  }
  std::vector<std::vector<Pending>> slots(n_slots);

  for (int c = 0; c < n_classes; ++c) {
    const muon_ns_class& k = classes[c];
    ClassGeom G{&k, op_dtype, es, std::min(k.rows, k.cols), std::max(k.rows, k.cols), k.rows <= k.cols,
                static_cast<long long>(k.rows) * k.ld_x, static_cast<long long>(std::min(k.rows, k.cols)) * k.ld_m};
    // The first iteration applies the per-matrix input scale unless x0 already
    // holds the normalised fp16 input (fp16 without MUON_NS_INPUT_SCALED).
    const bool scaled_in = !f16 || (k.flags & MUON_NS_INPUT_SCALED) != 0;
    auto xscale = [&](int it) { return ns_operand_scale(k.rows, k.cols, it, op_dtype); };
    if (k.algo == MUON_NS_STANDARD) {
      for (int it = 0; it < steps; ++it) {
        const void* xin = (it % 2 == 0) ? k.x0 : k.x1;
        const void* xout = (it % 2 == 0) ? k.x1 : k.x0;
        const bool last = it == steps - 1;
        // fp16: X is stored pre-normalised and scaled by S_it, so A = acc / S_it^2.
        const float S = xscale(it);
        slots[slot_of[3 * it]].push_back(G.gram_x(xin, scaled_in && it == 0, 1.0f / (S * S), nullptr, 1.0f));
        slots[slot_of[3 * it + 1]].push_back(G.sym(k.ap, k.bp, EPI_POLY, 1.0f, k.mm));
        // acc = M (S_it X): rescale to S_{it+1} X' for the next iteration, or to X' itself.
        const float Sn = last ? 1.0f : xscale(it + 1);
        slots[slot_of[3 * it + 2]].push_back(G.apply(k.mm, xin, scaled_in && it == 0, Sn / S, last ? nullptr : xout));
      }
      continue;
    }
    const float SA = gram_scale_a(G.m, op_dtype), SQ = gram_scale_q(G.m, op_dtype);
    for (int s0 = 0; s0 < steps; s0 += kGramSegment) {
      const int s1 = std::min(s0 + kGramSegment, steps);
      const int seg = s0 / kGramSegment;
      const void* xseg = (seg % 2 == 0) ? k.x0 : k.x1;
      const void* xnext = (seg % 2 == 0) ? k.x1 : k.x0;
      const float S = xscale(s0);
      auto qbuf = [&](int j) { return ((j - s0) % 2 == 0) ? k.qa : k.qb; };
      for (int it = s0; it < s1; ++it) {
        // phase 0: A' and B' of A_it, and A_it * SA
        if (it == s0)
          slots[slot_of[3 * it]].push_back(G.gram_x(xseg, scaled_in && it == 0, 1.0f / (S * S), k.aa, SA));
        else  // A_it = P_{it-1} (P_{it-1} A_{it-1}), operands stored times SA
          slots[slot_of[3 * it]].push_back([&] {
            Pending p = G.sym(k.mm, k.pa, EPI_GRAM, 1.0f / (SA * SA), k.ap);
            p.o2 = G.mat_out(k.bp);
            p.o3 = G.mat_out(k.aa);
            p.pr.omul3 = SA;
            return p;
          }());
        // phase 1: P_it = alpha I + A' B', stored times SA (and as Q times SQ
        // at the start of a segment)
        {
          Pending p = G.sym(k.ap, k.bp, EPI_POLY, 1.0f, k.mm);
          p.pr.omul = SA;
          if (it == s0) {
            p.o3 = G.mat_out(qbuf(it));
            p.pr.omul3 = SQ;
          }
          slots[slot_of[3 * it + 1]].push_back(p);
        }
        // phase 2: P A (for the next A) and Q_it = P_it Q_{it-1}
        if (it < s1 - 1) {
          Pending p = G.sym(k.mm, k.aa, EPI_APPLY, 1.0f / SA, k.pa);
          slots[slot_of[3 * it + 2]].push_back(p);
        }
        if (it > s0) {
          Pending p = G.sym(k.mm, qbuf(it - 1), EPI_APPLY, 1.0f / SA, qbuf(it));
          slots[slot_of[3 * it + 2]].push_back(p);
        }
      }
      // segment end: X_{s1} = Q X_{s0} (or U)
      const bool last = s1 == steps;
      const float Sn = last ? 1.0f : xscale(s1);
      slots[ex_slot[s1 - 1]].push_back(G.apply(qbuf(s1 - 1), xseg, scaled_in && s0 == 0, Sn / (SQ * S),
                                               last ? nullptr : xnext));
    }
  }

  muon_ns_plan* plan = new muon_ns_plan();
  plan->op_dtype = op_dtype;
  plan->steps = steps;
  plan->n_classes = n_classes;
  plan->num_sms = sms;
  const float alpha = float(kNsA + kNsB + kNsC);
  const float beta = float(kNsB + 2.0 * kNsC);
  const float gamma = float(kNsC);
  for (auto& list : slots) {
    if (list.empty()) continue;
    // Order problems by K (largest first) so long tiles start early.
    std::stable_sort(list.begin(), list.end(), [](const Pending& x, const Pending& y) {
      if (x.pr.K != y.pr.K) return x.pr.K > y.pr.K;
      return x.work > y.work;
    });
    plan->launches.emplace_back();
    GemmParams& L = plan->launches.back();
    memset(&L, 0, sizeof(L));
    L.alpha = alpha;
    L.beta = beta;
    L.gamma = gamma;
    int tile_begin = 0;
    for (size_t pi = 0; pi < list.size(); ++pi) {
      const int rc = encode_pending(L, static_cast<int>(pi), list[pi], op_dtype);
      if (rc != MUON_OK) {
        delete plan;
        return rc;
      }
      GemmProblem& pr = L.prob[pi];
      pr.tiles_per_mat = tiles_per_matrix(pr.M, pr.N, pr.symmetric != 0, &pr.tiles_m, &pr.tiles_n);
      pr.tile_begin = tile_begin;
      tile_begin += pr.tiles_per_mat * pr.batch;
    }
    L.n_problems = static_cast<int>(list.size());
    L.total_tiles = tile_begin;
  }
  *plan_out = plan;
  return MUON_OK;
}

int ns_plan_set_sm_limit(muon_ns_plan* plan, int sms) {
  if (!plan) return set_error(MUON_ERR_ARG, "plan is null");
  if (sms < 0) return set_error(MUON_ERR_ARG, "sm limit must be >= 0");
  if (sms != 0 && sms < 2) return set_error(MUON_ERR_ARG, "sm limit must leave at least one CTA pair (2 SMs)");
  plan->sm_limit = sms;
  return MUON_OK;
}

int ns_plan_run(const muon_ns_plan* plan, int* err_dev, cudaStream_t stream) {
  if (!plan) return set_error(MUON_ERR_ARG, "plan is null");
  if (!err_dev) return set_error(MUON_ERR_ARG, "err_dev is null");
  constexpr int kMaxDevices = 64;
  static std::mutex attr_mu;
  static int max_clusters[kMaxDevices][3] = {};  // per kernel (tf32, bf16, f16); 0: not set up yet
  const int op = plan->op_dtype;
  const int kern = op == MUON_TF32 ? 0 : op == MUON_BF16 ? 1 : 2;  // fp16 and split fp16 share a kernel
  const void* fn = op == MUON_TF32   ? reinterpret_cast<const void*>(&ns_gemm_kernel<kOpTf32>)
                   : op == MUON_BF16 ? reinterpret_cast<const void*>(&ns_gemm_kernel<kOpBf16>)
                                     : reinterpret_cast<const void*>(&ns_gemm_kernel<kOpF16>);
  int dev = 0;
  if (check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return MUON_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return set_error(MUON_ERR_UNSUPPORTED, "device ordinal above 63");
  int clusters = 0;
  {
  std::lock_guard<std::mutex> lock(attr_mu);
  if (max_clusters[dev][kern] == 0) {
    if (check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES),
                   "cudaFuncSetAttribute(ns_gemm)"))
      return MUON_ERR_CUDA;
    // Persistent schedule: launch only as many CTA pairs as can be resident
    // at once (a GPC with an odd number of free SMs leaves one unused).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (plan->num_sms / 2));
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int resident = 0;
    if (check_cuda(cudaOccupancyMaxActiveClusters(&resident, fn, &cfg), "cudaOccupancyMaxActiveClusters"))
      return MUON_ERR_CUDA;
    max_clusters[dev][kern] = std::max(1, std::min(resident, plan->num_sms / 2));
  }
  clusters = max_clusters[dev][kern];
  }
  if (plan->sm_limit > 0) clusters = std::max(1, std::min(clusters, plan->sm_limit / 2));
  const int n = static_cast<int>(plan->launches.size());
  for (int i = 0; i < n; ++i) {
    GemmParams L = plan->launches[i];
    L.err = err_dev;
    if (L.total_tiles == 0) continue;
    const int grid = 2 * std::min(L.total_tiles, clusters);  // CTA pairs
    if (op == MUON_TF32)
      ns_gemm_kernel<kOpTf32><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(L);
    else if (op == MUON_BF16)
      ns_gemm_kernel<kOpBf16><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(L);
    else
      ns_gemm_kernel<kOpF16><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(L);
    if (check_cuda(cudaGetLastError(), "ns_gemm launch")) return MUON_ERR_CUDA;
  }
  return MUON_OK;
}

void ns_plan_destroy(muon_ns_plan* plan) { delete plan; }

int ns_plan_launches(const muon_ns_plan* plan) {
  if (!plan) return -1;
  int n = 0;
  for (const auto& L : plan->launches) n += L.total_tiles > 0 ? 1 : 0;
  return n;
}

}  // namespace muon
