// Persistent warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M, N] = epilogue( sum_k A[m, k] * B[n, k] )
//
// Operands are bf16, staged global -> SMEM by TMA (128-byte swizzle, no cluster
// fan-out), multiplied by tcgen05.mma (M=128, N=BN, K=16) into an fp32 accumulator in
// TMEM.  Two TMEM accumulators alternate between tiles so the epilogue of tile i runs
// while the MMAs of tile i+1 are issued.
//
// Operand majors:
//   K-major  : the operand is stored [rows, K] row-major (nn.Linear weight, activations)
//   MN-major : the operand is stored [K, rows] row-major (dgrad B = W, wgrad A = dY, B = X)
// so forward (X W^T), dgrad (dY W) and wgrad (dY^T X) all run on the same kernel.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer,
// warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4) .. +32, one row per thread).
//
// The epilogue is a template functor `Epi` (one copy per thread) with
//   begin_tile()                                   before the chunks of a tile
//   apply(row, col0, ncols_valid, float (&v)[32], tile_n)   per valid 32-column chunk
//   end_tile(row, tile_n)                          after the chunks (rows < M only)
//   finish()                                       once, after the last tile
// Each epilogue thread owns one accumulator row per tile; rows >= M are skipped.
#pragma once
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "octo_api.h"

namespace octo {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kGemmThreads = 192;
constexpr int kGemmGroupM = 16;  // tile raster: 16 M-blocks share each B tile in L2

// MT = M-tiles per CTA: with MT = 2 a CTA multiplies two 128-row A tiles by each B tile it
// loads (decode-sized M), so every weight byte crosses L2 -> SMEM once instead of once per
// M-tile.  The accumulators take MT * BN TMEM columns; they are double-buffered when two
// sets fit the 512 columns, else single-buffered (a CTA then waits for its epilogue before
// the next tile's MMAs, which decode shapes with ~one tile per CTA never do).
template <int BN, int MT = 1>
struct GemmCfg {
  static_assert(MT == 1 || MT == 2, "one or two M-tiles per CTA");
  static constexpr int kAccCols = MT * BN;
  static constexpr int kAccBufs = 2 * kAccCols <= 512 ? 2 : 1;
  static constexpr int kStages = MT == 1 ? (BN == 256 ? 4 : (BN == 128 ? 6 : 8)) : (BN == 256 ? 3 : (BN == 128 ? 4 : 5));
  static constexpr int kATileBytes = kGemmBM * kGemmBK * 2;
  static constexpr int kABytes = MT * kATileBytes;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = kAccBufs * kAccCols < 32 ? 32 : kAccBufs * kAccCols;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(kSmemBytes <= 227 * 1024, "stage ring exceeds shared memory");
};


// K range of a tile's split: [kb0, kb1) in 64-wide K blocks
__device__ __forceinline__ void gemm_split_range(const GemmShape& s, int ks, int& kb0, int& kb1) {
  const int splits = s.k_splits > 1 ? s.k_splits : 1;
  const int per = (s.k_blocks + splits - 1) / splits;
  kb0 = min(s.k_blocks, ks * per);
  kb1 = min(s.k_blocks, kb0 + per);
}

// tile -> (M-block, N-block, K split); splits are the slowest index so CTAs running at the
// same time share their K slice of A in L2
__device__ __forceinline__ void gemm_tile_coords(const GemmShape& s, int tile, int& mb, int& nb, int& ks) {
  const int per_split = s.m_tiles * s.n_tiles;
  ks = tile / per_split;
  tile -= ks * per_split;
  const int group_span = kGemmGroupM * s.n_tiles;
  const int group = tile / group_span;
  const int first_m = group * kGemmGroupM;
  int gm = s.m_tiles - first_m;
  gm = gm < kGemmGroupM ? gm : kGemmGroupM;
  const int r = tile - group * group_span;
  mb = first_m + r % gm;
  nb = r / gm;
  if (s.m_shift) mb = (mb + s.m_shift) % s.m_tiles;
}

// An epilogue with `static constexpr bool kPaired = true` takes the two halves of a paired
// B tile (shape.b_pair > 0) together: apply_pair(row, col0, nvalid, lo[32], hi[32]) per
// 32-column chunk of the tile's BN / 2 output columns.
template <class E, class = void>
struct EpiPaired : std::false_type {};
template <class E>
struct EpiPaired<E, std::void_t<decltype(E::kPaired)>> : std::bool_constant<E::kPaired> {};

// ---------------------------------------------------------------- A-operand sources
//
// The producer asks its A source for the bytes of an M-block (the stage's expect-tx
// count) and to issue the TMA loads of one (M-block, K-block) tile.  `signal()` runs
// once per CTA before any wait, `finish_cta()` once per CTA after the last use.

// One tensor map over a local matrix (K-major: [M, K]; MN-major: [K, M]).
template <bool A_MN>
struct ALocal {
  CUtensorMap m;
  __device__ __forceinline__ void prefetch() const { tma_prefetch_desc(&m); }
  __device__ __forceinline__ void signal() const {}
  __device__ __forceinline__ void finish_cta() const {}
  __device__ __forceinline__ void prologue(int, volatile int*, int*) const {}
  __device__ __forceinline__ bool ready(int, uint32_t&, volatile int*, int*) const { return true; }
  __device__ __forceinline__ uint32_t bytes(int) const { return kGemmBM * kGemmBK * 2; }
  __device__ __forceinline__ void load(uint8_t* dst, uint64_t* bar, int k0, int mb) const {
    const int m0 = mb * kGemmBM;
    if constexpr (!A_MN) {
      tma_load_2d(dst, &m, bar, k0, m0);
    } else {
#pragma unroll
      for (int j = 0; j < kGemmBM / 64; ++j) tma_load_2d(dst + j * 8192, &m, bar, m0 + 64 * j, k0);
    }
  }
};

template <int BN, bool A_MN, bool B_MN, class Epi, class ASrc = ALocal<A_MN>, int MT = 1>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ ASrc asrc_param, const __grid_constant__ CUtensorMap tmB,
                        GemmShape shape, Epi epi, int* status) {
  // (each thread works on its own copy of the epilogue functor; with MT = 2, shape.m_tiles
  // counts pairs of 128-row M-blocks and tile coordinate mb covers rows 256 mb .. +256)
  using Cfg = GemmCfg<BN, MT>;
  static_assert(MT == 1 || !A_MN, "two M-tiles per CTA take a K-major A");
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* accf_bar = empty_bar + S;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* drain_bar = acce_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf_bar[i], 1);
      mbar_init(&acce_bar[i], 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    asrc_param.prefetch();
    tma_prefetch_desc(&tmB);
    asrc_param.signal();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const ASrc& asrc = asrc_param;
      uint32_t ready_mask = 0;  // source ranks whose data this CTA has seen published
      // L2 prefetch cursor over this CTA's (tile, K-block) sequence, kept `ahead` K-blocks in
      // front of the TMA loads: weight tiles stream from DRAM into L2 with more bytes in flight
      // than the shared-memory ring holds, so the ring's loads hit L2.
      const int ahead = shape.b_prefetch > 0 ? shape.b_prefetch : (shape.pdl ? S : 0);
      int pf_tile = blockIdx.x, pf_nb = 0, pf_kb = 0, pf_kb1 = 0;
      auto pf_coords = [&]() {
        int mb_, ks_;
        gemm_tile_coords(shape, pf_tile, mb_, pf_nb, ks_);
        gemm_split_range(shape, ks_, pf_kb, pf_kb1);
      };
      auto pf_step = [&]() {  // prefetch one K-block of B, then advance the cursor
        if (pf_tile >= shape.num_tiles) return;
        if constexpr (!B_MN) {
          if (shape.b_pair > 0) {
            tma_prefetch_l2_2d(&tmB, pf_kb * kGemmBK, pf_nb * (BN / 2));
            tma_prefetch_l2_2d(&tmB, pf_kb * kGemmBK, shape.b_pair + pf_nb * (BN / 2));
          } else {
            tma_prefetch_l2_2d(&tmB, pf_kb * kGemmBK, pf_nb * BN);
          }
        } else {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) tma_prefetch_l2_2d(&tmB, pf_nb * BN + 64 * j, pf_kb * kGemmBK);
        }
        if (++pf_kb >= pf_kb1) {
          pf_tile += gridDim.x;
          if (pf_tile < shape.num_tiles) pf_coords();
        }
      };
      if (pf_tile < shape.num_tiles) pf_coords();
      // (a programmatic dependent issues these before waiting: B does not depend on the
      // preceding kernel)
      for (int i = 0; i < ahead; ++i) pf_step();
      if (shape.pdl) grid_dep_wait();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < shape.num_tiles && ok; tile += gridDim.x) {
        int mb, nb, ks, kb0, kb1;
        gemm_tile_coords(shape, tile, mb, nb, ks);
        gemm_split_range(shape, ks, kb0, kb1);
        const int n0 = nb * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, status, 100 + stage)) {
            ok = false;
            break;
          }
          const int k0 = kb * kGemmBK;
          uint8_t* a_dst = sA + stage * Cfg::kABytes;
          uint8_t* b_dst = sB + stage * Cfg::kBBytes;
          if (kb == kb0 && !asrc.ready(mb, ready_mask, abort_flag, status)) {  // peer data of this M-block published?
            ok = false;
            break;
          }
          if constexpr (MT == 1) {
            mbar_arrive_expect_tx(&full_bar[stage], asrc.bytes(mb) + Cfg::kBBytes);
            asrc.load(a_dst, &full_bar[stage], k0, mb);
          } else {
            mbar_arrive_expect_tx(&full_bar[stage], asrc.bytes(MT * mb) * MT + Cfg::kBBytes);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) asrc.load(a_dst + mt * Cfg::kATileBytes, &full_bar[stage], k0, MT * mb + mt);
          }
          if constexpr (!B_MN) {
            if (shape.b_pair > 0) {  // two half-height boxes (the map's box is BN / 2 rows)
              const int r0 = nb * (BN / 2);
              tma_load_2d(b_dst, &tmB, &full_bar[stage], k0, r0);
              tma_load_2d(b_dst + (BN / 2) * kGemmBK * 2, &tmB, &full_bar[stage], k0, shape.b_pair + r0);
            } else {
              tma_load_2d(b_dst, &tmB, &full_bar[stage], k0, n0);
            }
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full_bar[stage], n0 + 64 * j, k0);
          }
          if (shape.b_prefetch > 0) pf_step();
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Drain: wait (bounded) until every copy this thread issued has landed.
        const uint64_t t0 = globaltimer_ns();
        for (int s = 0; s < S; ++s) {
          if (!(issued_mask & (1u << s))) continue;
          while (!mbar_try_wait(&full_bar[s], (issued_parity >> s) & 1u)) {
            if (globaltimer_ns() - t0 > OCTO_WAIT_NS) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(kGemmBM, BN, A_MN, B_MN, true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = blockIdx.x; tile < shape.num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1u, abort_flag, status, 200 + acc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::kAccCols);
        int mb_, nb_, ks, kb0, kb1;
        gemm_tile_coords(shape, tile, mb_, nb_, ks);
        gemm_split_range(shape, ks, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, status, 300 + stage)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int kk = 0; kk < kGemmBK / 16; ++kk) {
            uint64_t da, db;
            if constexpr (!A_MN) {
              da = umma_smem_desc(a_addr + kk * 32, 16, 1024);
            } else {
              da = umma_smem_desc(a_addr + kk * 2048, 8192, 1024);
            }
            if constexpr (!B_MN) {
              db = umma_smem_desc(b_addr + kk * 32, 16, 1024);
            } else {
              db = umma_smem_desc(b_addr + kk * 2048, 8192, 1024);
            }
            const uint32_t accum = (kb != kb0 || kk != 0) ? 1u : 0u;
            umma_f16_ss(d_tmem, da, db, idesc, accum);
#pragma unroll
            for (int mt = 1; mt < MT; ++mt)  // further M-tiles reuse the B descriptor (K-major A only)
              umma_f16_ss(d_tmem + mt * BN, umma_smem_desc(a_addr + mt * Cfg::kATileBytes + kk * 32, 16, 1024), db,
                          idesc, accum);
          }
          issued_any = true;
          umma_commit(&empty_bar[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&accf_bar[acc]);
        if (++acc == Cfg::kAccBufs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        // Drain: all MMAs issued so far must finish before TMEM is released.
        umma_commit(drain_bar);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain_bar, 0)) {
          if (globaltimer_ns() - t0 > OCTO_WAIT_NS) break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    asrc_param.prologue(threadIdx.x - 64, abort_flag, status);  // (A-source staging work, if any)
    const int quarter = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < shape.num_tiles; tile += gridDim.x) {
      if (!mbar_wait(&accf_bar[acc], acc_phase, abort_flag, status, 400 + acc)) break;
      tc_fence_after();
      int mb, nb, ks, kb0, kb1;
      gemm_tile_coords(shape, tile, mb, nb, ks);
      gemm_split_range(shape, ks, kb0, kb1);
      const bool empty_k = kb1 <= kb0;  // no MMA wrote the accumulator: the tile's sum is 0
      const int n0 = nb * BN;
#pragma unroll 1
      for (int mt = 0; mt < MT; ++mt) {
        const int row = (MT * mb + mt) * kGemmBM + quarter * 32 + lane;
        epi.begin_split(ks);
        epi.begin_tile();
        if constexpr (EpiPaired<Epi>::value) {
          // paired tile: TMEM columns [0, BN/2) hold the first half, [BN/2, BN) the second
#pragma unroll 1
          for (int c = 0; c < BN / 64; ++c) {
            uint32_t r[32], r2[32];
            const uint32_t cb = tmem_base + lane_base + static_cast<uint32_t>(acc * Cfg::kAccCols + mt * BN + c * 32);
            tmem_ld_32x32b_x32(cb, r);
            tmem_ld_32x32b_x32(cb + BN / 2, r2);
            tmem_wait_ld();
            const int col0 = nb * (BN / 2) + c * 32;
            if (row < shape.M && col0 < shape.N) {
              float lo[32], hi[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                lo[i] = empty_k ? 0.f : __uint_as_float(r[i]);
                hi[i] = empty_k ? 0.f : __uint_as_float(r2[i]);
              }
              const int nvalid = shape.N - col0 < 32 ? shape.N - col0 : 32;
              epi.apply_pair(row, col0, nvalid, lo, hi);
            }
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + lane_base + static_cast<uint32_t>(acc * Cfg::kAccCols + mt * BN + c * 32), r);
            tmem_wait_ld();
            const int col0 = n0 + c * 32;
            if (row < shape.M && col0 < shape.N) {
              float v[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = empty_k ? 0.f : __uint_as_float(r[i]);
              const int nvalid = shape.N - col0 < 32 ? shape.N - col0 : 32;
              epi.apply(row, col0, nvalid, v, nb);
            }
          }
        }
        if (mt == MT - 1) {  // accumulator drained: the MMA warp may reuse it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce_bar[acc]);
        }
        if (row < shape.M) epi.end_tile(row, nb);
      }
      if (++acc == Cfg::kAccBufs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    epi.finish();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
  if (threadIdx.x == 0) asrc_param.finish_cta();
}

// ---------------------------------------------------------------- epilogues

// C (bf16, row stride ldc) = alpha * acc (+ bias[col]) (+ residual bf16, row stride ldr)
struct EpiBF16 {
  __nv_bfloat16* C;
  int ldc;
  const __nv_bfloat16* R;
  int ldr;
  float alpha;
  const __nv_bfloat16* bias;
  __device__ __forceinline__ void apply(int row, int col0, int nvalid, float (&v)[32], int) {
    __nv_bfloat16* dst = C + static_cast<size_t>(row) * ldc + col0;
    float a = alpha;  // local: the functor persists across chunks and tiles
    if (bias != nullptr) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        if (g * 8 < nvalid) {
          uint4 bv = *reinterpret_cast<const uint4*>(bias + col0 + g * 8);
          const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&bv);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[g * 8 + i] = v[g * 8 + i] * a + __bfloat162float(bb[i]);
        }
      }
      a = 1.0f;  // already applied
    }
    if (R != nullptr) {
      const __nv_bfloat16* res = R + static_cast<size_t>(row) * ldr + col0;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        if (g * 8 < nvalid) {
          uint4 rv = *reinterpret_cast<const uint4*>(res + g * 8);
          const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[g * 8 + i] = a * v[g * 8 + i] + __bfloat162float(rb[i]);
        }
      }
    } else if (a != 1.0f) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= a;
    }
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (g * 8 < nvalid) {
        uint4 o;
        o.x = pack_bf16x2(v[g * 8 + 0], v[g * 8 + 1]);
        o.y = pack_bf16x2(v[g * 8 + 2], v[g * 8 + 3]);
        o.z = pack_bf16x2(v[g * 8 + 4], v[g * 8 + 5]);
        o.w = pack_bf16x2(v[g * 8 + 6], v[g * 8 + 7]);
        *reinterpret_cast<uint4*>(dst + g * 8) = o;
      }
    }
  }
  __device__ __forceinline__ void begin_split(int) {}
  __device__ __forceinline__ void begin_tile() {}
  __device__ __forceinline__ void end_tile(int, int) {}
  __device__ __forceinline__ void finish() const {}
};

// C (fp32) = alpha * acc  (+ C if accumulate)
struct EpiF32 {
  float* C;
  int ldc;
  float alpha;
  int accumulate;
  __device__ __forceinline__ void apply(int row, int col0, int nvalid, float (&v)[32], int) {
    float* dst = C + static_cast<size_t>(row) * ldc + col0;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      if (g * 4 < nvalid) {
        float4 o = make_float4(alpha * v[g * 4], alpha * v[g * 4 + 1], alpha * v[g * 4 + 2], alpha * v[g * 4 + 3]);
        if (accumulate) {
          const float4 p = *reinterpret_cast<const float4*>(dst + g * 4);
          o.x += p.x;
          o.y += p.y;
          o.z += p.z;
          o.w += p.w;
        }
        *reinterpret_cast<float4*>(dst + g * 4) = o;
      }
    }
  }
  __device__ __forceinline__ void begin_split(int) {}
  __device__ __forceinline__ void begin_tile() {}
  __device__ __forceinline__ void end_tile(int, int) {}
  __device__ __forceinline__ void finish() const {}
};

// Gated MLP: C (bf16 [M, N], row stride ldc) = silu(gate) * up, where the paired tile's first
// half is the gate projection and its second half the up projection of the same N columns.
// Gate and up are rounded to bf16 first, so the result equals the unfused GEMM (bf16 output)
// followed by swiglu_fwd_kernel.
struct EpiSwiGLU {
  static constexpr bool kPaired = true;
  __nv_bfloat16* C;
  int ldc;
  __device__ __forceinline__ void apply_pair(int row, int col0, int nvalid, float (&g)[32], float (&u)[32]) {
    __nv_bfloat16* dst = C + static_cast<size_t>(row) * ldc + col0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (q * 8 < nvalid) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float gb = __bfloat162float(__float2bfloat16(g[q * 8 + i]));
          const float ub = __bfloat162float(__float2bfloat16(u[q * 8 + i]));
          o[i] = gb / (1.f + __expf(-gb)) * ub;
        }
        uint4 w;
        w.x = pack_bf16x2(o[0], o[1]);
        w.y = pack_bf16x2(o[2], o[3]);
        w.z = pack_bf16x2(o[4], o[5]);
        w.w = pack_bf16x2(o[6], o[7]);
        *reinterpret_cast<uint4*>(dst + q * 8) = w;
      }
    }
  }
  __device__ __forceinline__ void apply(int, int, int, float (&)[32], int) {}
  __device__ __forceinline__ void begin_split(int) {}
  __device__ __forceinline__ void begin_tile() {}
  __device__ __forceinline__ void end_tile(int, int) {}
  __device__ __forceinline__ void finish() const {}
};

// QKV projection with the rotary embedding (training forward): tile nb is head nb (BN = head
// dim D), so the paired halves of a chunk are the rotary pairs (i, i + D/2) of one head.
// C (bf16, row stride ldc) = acc + bias, rounded to bf16, then rotated by pos[row] on the
// q and k heads in fp32 and rounded again - the unfused GEMM (bf16 output) + rope_kernel.
struct EpiQKVRope {
  static constexpr bool kPaired = true;
  __nv_bfloat16* C;
  int ldc;
  const __nv_bfloat16* bias;
  const int32_t* pos;
  float log2_theta;
  int rot_heads;
  int D;
  __device__ __forceinline__ void apply_pair(int row, int col0, int, float (&lo)[32], float (&hi)[32]) {
    const int half = D >> 1;
    const int h = col0 / half;          // head (= tile)
    const int i0 = col0 - h * half;     // rotary index of lo[0]
    const int clo = h * D + i0, chi = clo + half;
    if (bias != nullptr) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float bl[8], bh[8];
        load8(bias + clo + q * 8, bl);
        load8(bias + chi + q * 8, bh);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          lo[q * 8 + i] += bl[i];
          hi[q * 8 + i] += bh[i];
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      lo[i] = __bfloat162float(__float2bfloat16(lo[i]));
      hi[i] = __bfloat162float(__float2bfloat16(hi[i]));
    }
    if (h < rot_heads) {
      const int p = pos[row];
#pragma unroll 4
      for (int i = 0; i < 32; ++i) {
        float sn, cs;
        rope_sincos(p, i0 + i, D, log2_theta, sn, cs);
        const float a = lo[i], b = hi[i];
        lo[i] = a * cs - b * sn;
        hi[i] = b * cs + a * sn;
      }
    }
    __nv_bfloat16* dl = C + static_cast<size_t>(row) * ldc + clo;
    __nv_bfloat16* dh = C + static_cast<size_t>(row) * ldc + chi;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float tl[8], th[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        tl[i] = lo[q * 8 + i];
        th[i] = hi[q * 8 + i];
      }
      store8(dl + q * 8, tl);
      store8(dh + q * 8, th);
    }
  }
  __device__ __forceinline__ void apply(int, int, int, float (&)[32], int) {}
  __device__ __forceinline__ void begin_split(int) {}
  __device__ __forceinline__ void begin_tile() {}
  __device__ __forceinline__ void end_tile(int, int) {}
  __device__ __forceinline__ void finish() const {}
};

// fp32 partial of K split `ks` -> ws[ks][row][col] (row stride N); a finish kernel sums the splits
struct EpiSplitK {
  float* ws;
  int M, N;
  float* cur;
  __device__ __forceinline__ void begin_split(int ks) { cur = ws + static_cast<size_t>(ks) * M * N; }
  __device__ __forceinline__ void begin_tile() {}
  __device__ __forceinline__ void apply(int row, int col0, int nvalid, float (&v)[32], int) {
    float* dst = cur + static_cast<size_t>(row) * N + col0;
#pragma unroll
    for (int g = 0; g < 8; ++g)
      if (g * 4 < nvalid) *reinterpret_cast<float4*>(dst + g * 4) = make_float4(v[g * 4], v[g * 4 + 1], v[g * 4 + 2], v[g * 4 + 3]);
  }
  __device__ __forceinline__ void end_tile(int, int) {}
  __device__ __forceinline__ void finish() const {}
};

}  // namespace octo
