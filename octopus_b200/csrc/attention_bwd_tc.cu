// Gathered-key attention backward on tcgen05/TMEM (head_dim 128), two kernels:
//
//   dq kernel   CTA = 128 query rows of one sequence x one query head; walks the key tiles:
//                 S = Q K_j^T, dP = dO V_j^T          (tcgen05.mma, SMEM operands, fp32 TMEM)
//                 dS = P o (dP - delta), P = exp(S scale - lse)   (thread = query row)
//                 dQ += dS K_j                         (A = dS in TMEM as bf16, over S)
//   dkv kernel  CTA = 128 key rows of one sequence x one KV head; walks (query head of the
//               GQA group, 64-row query sub-tile) steps:
//                 S^T = K Q_i^T, dP^T = V dO_i^T       (M = 128 keys, N = 64 queries)
//                 P^T, dS^T                            (thread = key row)
//                 dV += P^T dO_i, dK += dS^T Q_i       (A from TMEM, over S^T / dP^T)
//               and scatter-adds dK (x scale), dV into the fp32 accumulators of the
//               gathered key rows (a key row is shared by the tree paths through it).
// dQ needs no atomics: it is recomputed per query tile (7 MMAs per tile pair in all
// instead of 5 plus an fp32 reduction of every dQ partial).
//
// Warp roles (both kernels, 384 threads): warp 0 streams the operand whose rows are
// contiguous (Q/dO, TMA), warp 1 owns TMEM and issues the MMAs from an event loop, warps 2-3
// load the gathered key rows (two TMA boxes per 64 rows when consecutive in the key list,
// cp.async otherwise), warps 4-7 and 8-11 (two per SM sub-partition, hiding each other's
// TMEM and MUFU latency) do the elementwise work on the two column halves and the epilogue.
//
// TMEM: dq kernel  S[0] [0,128), S[1] [128,256), dP [256,384), dQ [384,512); the bf16 dS
//                  of key half w goes to S columns [64w, 64w + 32) (inside that half's own S
//                  range, so neither half overwrites columns the other still reads)
//       dkv kernel S^T[0] [0,64), S^T[1] [64,128), dP^T[0] [128,192), dP^T[1] [192,256),
//                  dV [256,384), dK [384,512); P^T / dS^T of query half w at [32w, 32w + 16)
//                  of their buffer
// All waits are bounded (common.cuh); a timed-out CTA records an error, drains and frees TMEM.
//
// Reference parity (behaviour): gradients of the tree attention the reference trains through
// `octopus/rl/prefix_tree.py` (FlashAttention-2 style backward: delta = rowsum(dO o O)).
#include <cuda.h>
#include <cuda_bf16.h>

#include "attention.h"
#include "common.cuh"

namespace octo {

namespace {

constexpr int kD = 128;
constexpr int kHalf = 128 * 128;   // 64-column SW128 half of a 128-row tile
constexpr int kTile = 2 * kHalf;   // 32 KB
constexpr int kHalf64 = 64 * 128;  // 64-column half of a 64-row tile
constexpr int kTile64 = 2 * kHalf64;
constexpr int kThreads = 384;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t toff(int r, int c) {
  return static_cast<uint32_t>((c >> 3) * kHalf + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Loads this warp's 64 rows (tile rows rbase..rbase+63) of a gathered K or V tile: two TMA
// boxes (64 rows x 64 columns each) when the rows are consecutive, else cp.async.  Every
// lane arrives once on `bar` (count 64 over the two producer warps).
__device__ __forceinline__ void load_gathered(uint8_t* dst, const CUtensorMap* map, const __nv_bfloat16* src,
                                              int ldk, uint64_t* bar, int rbase, int col0, bool contig, int base,
                                              const int (&ix)[2]) {
  const int lane = threadIdx.x & 31;
  if (contig) {
    if (lane == 0) {
      mbar_arrive_expect_tx(bar, 2u * 64u * 128u);
#pragma unroll
      for (int half = 0; half < 2; ++half) tma_load_2d(dst + half * kHalf + rbase * 128, map, bar, col0 + half * 64, base);
    } else {
      mbar_arrive(bar);
    }
  } else {
    const int cl = lane & 15;
    const uint32_t sbase = smem_u32(dst);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int rl = 2 * i + (lane >> 4);
      const int64_t row = static_cast<int64_t>(__shfl_sync(0xffffffffu, ix[rl >> 5], rl & 31));
      cp_async16(sbase + toff(rbase + rl, cl), src + row * ldk + cl * 8);
    }
    cp_async_arrive(bar);
  }
}

// Key-list indices of this warp's rows of key tile j (rows past n_end read `first`) and
// whether they are consecutive (rows < n_end only).
__device__ __forceinline__ bool gather_rows(const int32_t* kidx, int j, int rbase, int n_end, int first,
                                            int (&ix)[2], int& base) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int kk = j * 128 + rbase + q * 32 + lane;
    ix[q] = kk < n_end ? static_cast<int>(kidx[kk]) : first;
  }
  base = __shfl_sync(0xffffffffu, ix[0], 0);
  bool c = true;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int kk = j * 128 + rbase + q * 32 + lane;
    if (kk < n_end && ix[q] != base + q * 32 + lane) c = false;
  }
  return __all_sync(0xffffffffu, c);
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          int where) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, status, where);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// dS = P o (dP - delta) of 32 keys (key index k0 + i; keys >= lim masked), packed bf16 pairs
__device__ __forceinline__ void ds_chunk(const uint32_t (&sv)[32], const uint32_t (&dv)[32], int k0, int lim,
                                         float sc, float lse2, float dlt, uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int k = k0 + 2 * i;
    const float p0 = k < lim ? exp2_approx(fmaf(__uint_as_float(sv[2 * i]), sc, -lse2)) : 0.f;
    const float p1 = k + 1 < lim ? exp2_approx(fmaf(__uint_as_float(sv[2 * i + 1]), sc, -lse2)) : 0.f;
    pk[i] = pack_bf16x2(p0 * (__uint_as_float(dv[2 * i]) - dlt), p1 * (__uint_as_float(dv[2 * i + 1]) - dlt));
  }
}

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > OCTO_WAIT_NS) break;
}

}  // namespace

// =============================================================================== dQ
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_dq_tc_kernel(const __grid_constant__ AttnBwdMaps maps, AttnBwdParams p, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = smem;
  uint8_t* sdO = sQ + kTile;
  uint8_t* sK = sdO + kTile;      // [2]
  uint8_t* sV = sK + 2 * kTile;   // [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * kTile);
  uint64_t* qd_full = bars;
  uint64_t* k_full = qd_full + 1;    // [2]
  uint64_t* v_full = k_full + 2;     // [2]
  uint64_t* k_empty = v_full + 2;    // [2]
  uint64_t* v_empty = k_empty + 2;   // [2]
  uint64_t* s_full = v_empty + 2;    // [2]
  uint64_t* dq_done = s_full + 2;    // [2] (per S buffer)
  uint64_t* dp_full = dq_done + 2;
  uint64_t* dp_free = dp_full + 1;
  uint64_t* ds_full = dp_free + 1;   // [2] (per S buffer)
  uint64_t* drain = ds_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr uint32_t kColDP = 256, kColDQ = 384;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x / p.Hq;
  const int h = blockIdx.x - tile * p.Hq;
  const int seq = p.tiles[2 * tile];
  const int q0 = p.tiles[2 * tile + 1];
  const int kvh = h / (p.Hq / p.Hkv);
  const int qbeg = p.cu_q[seq], nq = p.cu_q[seq + 1] - qbeg;
  const int kbeg = p.cu_k[seq], nk = p.cu_k[seq + 1] - kbeg;
  const int off = nk - nq;
  const int mrows = min(128, nq - q0);
  const int n_end = max(0, p.causal ? min(nk, q0 + mrows + off) : nk);
  const int nt = (n_end + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(qd_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 64);
      mbar_init(&v_full[s], 64);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&dq_done[s], 1);
    }
    mbar_init(dp_full, 1);
    mbar_init(dp_free, 8);
    mbar_init(&ds_full[0], 8);
    mbar_init(&ds_full[1], 8);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&maps.q);
    tma_prefetch_desc(&maps.dO);
    tma_prefetch_desc(&maps.k);
    tma_prefetch_desc(&maps.v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && nt > 0) {
      mbar_arrive_expect_tx(qd_full, 2u * kTile);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int rb = 0; rb < 2; ++rb) {
          const int c0 = h * kD + half * 64, r0 = qbeg + q0 + rb * 64;
          tma_load_2d(sQ + half * kHalf + rb * 8192, &maps.q, qd_full, c0, r0);
          tma_load_2d(sdO + half * kHalf + rb * 8192, &maps.dO, qd_full, c0, r0);
        }
      }
      drain_wait(qd_full, 0);
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ K / V producers
    const int rbase = (warp - 2) * 64;
    const int32_t* kidx = p.key_idx + kbeg;
    const int first = nk > 0 ? kidx[0] : 0;
    const __nv_bfloat16* kb = p.k + static_cast<size_t>(kvh) * kD;
    const __nv_bfloat16* vb = p.v + static_cast<size_t>(kvh) * kD;
    int last_k = -1, last_v = -1;
    bool ok = true;
    for (int j = 0; j < nt && ok; ++j) {
      const int st = j & 1;
      const uint32_t ph = static_cast<uint32_t>((j >> 1) & 1);
      int ix[2], base;
      const bool contig = gather_rows(kidx, j, rbase, n_end, first, ix, base);
      if (!(ok = warp_wait(&k_empty[st], ph ^ 1u, abort_flag, status, 900 + st))) break;
      load_gathered(sK + st * kTile, &maps.k, kb, p.ldk, &k_full[st], rbase, kvh * kD, contig, base, ix);
      last_k = j;
      if (!(ok = warp_wait(&v_empty[st], ph ^ 1u, abort_flag, status, 910 + st))) break;
      load_gathered(sV + st * kTile, &maps.v, vb, p.ldk, &v_full[st], rbase, kvh * kD, contig, base, ix);
      last_v = j;
    }
    if (!ok) {
      asm volatile("cp.async.wait_all;" ::: "memory");
      if (lane == 0) {
        for (int j = max(0, last_k - 1); j <= last_k; ++j) drain_wait(&k_full[j & 1], (j >> 1) & 1);
        for (int j = max(0, last_v - 1); j <= last_v; ++j) drain_wait(&v_full[j & 1], (j >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (event loop)
    if (lane == 0 && nt > 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(128, 128, false, false, true);
      constexpr uint32_t idesc_q = umma_idesc_f16(128, kD, false, true, true);
      bool ok = mbar_wait(qd_full, 0, abort_flag, status, 920);
      int js = 0, jd = 0, jq = 0;
      bool issued = false;
      uint64_t t_last = globaltimer_ns();
      const uint32_t qaddr = smem_u32(sQ), doaddr = smem_u32(sdO);
      while (ok && jq < nt) {
        bool progressed = false;
        // S(js) = Q K_js^T into S[js & 1]: needs K_js and dQ(js - 2) (the buffer's last reader) complete
        if (js < nt && mbar_test(&k_full[js & 1], (js >> 1) & 1) &&
            (js < 2 || mbar_test(&dq_done[js & 1], ((js - 2) >> 1) & 1))) {
          tc_fence_after();
          fence_proxy_async_smem();
          const uint32_t kaddr = smem_u32(sK + (js & 1) * kTile);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t o16 = (kk >> 2) * kHalf + (kk & 3) * 32;
            umma_f16_ss(tmem + (js & 1) * 128, umma_smem_desc(qaddr + o16, 16, 1024),
                        umma_smem_desc(kaddr + o16, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[js & 1]);
          ++js;
          issued = progressed = true;
        }
        // dP(jd) = dO V_jd^T: needs V_jd and dP(jd - 1) read by the elementwise warps (issued
        // before the pending dQ so the next tile's elementwise work can start sooner)
        if (jd < js && mbar_test(&v_full[jd & 1], (jd >> 1) & 1) &&
            (jd == 0 || mbar_test(dp_free, (jd - 1) & 1))) {
          tc_fence_after();
          fence_proxy_async_smem();
          const uint32_t vaddr = smem_u32(sV + (jd & 1) * kTile);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t o16 = (kk >> 2) * kHalf + (kk & 3) * 32;
            umma_f16_ss(tmem + kColDP, umma_smem_desc(doaddr + o16, 16, 1024), umma_smem_desc(vaddr + o16, 16, 1024),
                        idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(dp_full);
          umma_commit(&v_empty[jd & 1]);
          ++jd;
          issued = progressed = true;
        }
        // dQ += dS(jq) K_jq (dS of key half w at S columns [64w, 64w + 32))
        if (jq < jd && mbar_test(&ds_full[jq & 1], (jq >> 1) & 1)) {
          tc_fence_after();
          const uint32_t kaddr = smem_u32(sK + (jq & 1) * kTile);
#pragma unroll
          for (int kk = 0; kk < 128 / 16; ++kk) {
            const uint64_t bd = umma_smem_desc(kaddr + kk * 2048, kHalf, 1024);
            const uint32_t acol = (jq & 1) * 128 + (kk >> 2) * 64 + (kk & 3) * 8;
            umma_f16_ts(tmem + kColDQ, tmem + acol, bd, idesc_q, (jq > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&dq_done[jq & 1]);
          umma_commit(&k_empty[jq & 1]);
          ++jq;
          issued = progressed = true;
        }
        if (progressed) {
          t_last = globaltimer_ns();
        } else if (*abort_flag) {
          ok = false;
        } else if (globaltimer_ns() - t_last > wait_budget_ns(status)) {
          *abort_flag = 1;
          record_error(status, kErrMbarTimeout, 930);
          ok = false;
        }
      }
      if (issued) {
        umma_commit(drain);
        drain_wait(drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ dS + epilogue (thread = query row)
    const int quarter = warp & 3;
    const int wh = (warp - 4) >> 2;             // key half of every tile: [64 wh, 64 wh + 64)
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const bool valid = r < mrows;
    const int qi = q0 + r;
    const int lim = valid ? (p.causal ? min(n_end, qi + off + 1) : n_end) : 0;
    const float sc = p.scale * kLog2e;
    const float lse2 = valid ? p.lse[static_cast<size_t>(h) * p.Tq + qbeg + qi] * kLog2e : 0.f;
    const float dlt = valid ? p.delta[static_cast<size_t>(h) * p.Tq + qbeg + qi] : 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const uint32_t colS = (j & 1) * 128 + wh * 64;
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, abort_flag, status, 940) ||
          !mbar_wait(dp_full, j & 1, abort_flag, status, 941)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t d0[32], d1[32], sv[32];
      tmem_ld_32x32b_x32(tmem + lane_addr + kColDP + wh * 64, d0);
      tmem_ld_32x32b_x32(tmem + lane_addr + kColDP + wh * 64 + 32, d1);
      tmem_ld_32x32b_x32(tmem + lane_addr + colS, sv);
      tmem_wait_ld();
      // this half of dP is in registers: the next dP may be issued
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dp_free);
      const int kbase = j * 128 + wh * 64;
      uint32_t pk[16];
      ds_chunk(sv, d0, kbase, lim, sc, lse2, dlt, pk);
      // dS chunk c -> columns [16c, 16c + 16) of this half's S range (columns < 32(c + 1) of
      // the range are already in registers)
      tmem_st_32x32b_x16(tmem + lane_addr + colS, pk);
      tmem_ld_32x32b_x32(tmem + lane_addr + colS + 32, sv);
      tmem_wait_ld();
      ds_chunk(sv, d1, kbase + 32, lim, sc, lse2, dlt, pk);
      tmem_st_32x32b_x16(tmem + lane_addr + colS + 16, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[j & 1]);
    }
    const int last = nt - 1;
    __nv_bfloat16* dqrow = p.dq + static_cast<size_t>(qbeg + q0 + (valid ? r : 0)) * p.lddq +
                           static_cast<size_t>(h) * kD + wh * 64;
    if (ok && nt > 0 && mbar_wait(&dq_done[last & 1], (last >> 1) & 1, abort_flag, status, 950)) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + kColDQ + wh * 64 + c * 32, v);
        tmem_wait_ld();
        if (valid) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(v[g * 8 + 0]) * p.scale, __uint_as_float(v[g * 8 + 1]) * p.scale);
            u.y = pack_bf16x2(__uint_as_float(v[g * 8 + 2]) * p.scale, __uint_as_float(v[g * 8 + 3]) * p.scale);
            u.z = pack_bf16x2(__uint_as_float(v[g * 8 + 4]) * p.scale, __uint_as_float(v[g * 8 + 5]) * p.scale);
            u.w = pack_bf16x2(__uint_as_float(v[g * 8 + 6]) * p.scale, __uint_as_float(v[g * 8 + 7]) * p.scale);
            *reinterpret_cast<uint4*>(dqrow + c * 32 + g * 8) = u;
          }
        }
      }
    } else if (nt == 0 && valid) {
      for (int c = 0; c < 64; c += 8) *reinterpret_cast<uint4*>(dqrow + c) = make_uint4(0, 0, 0, 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ============================================================================== dK dV
constexpr int kQStages = 4;

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_dkv_tc_kernel(const __grid_constant__ AttnBwdMaps maps, AttnBwdParams p, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sK = smem;
  uint8_t* sV = sK + kTile;
  uint8_t* sQ = sV + kTile;                  // [kQStages] 64-row tiles
  uint8_t* sdO = sQ + kQStages * kTile64;    // [kQStages]
  float* sL = reinterpret_cast<float*>(sdO + kQStages * kTile64);  // [kQStages][64] lse
  float* sDl = sL + kQStages * 64;                                 // [kQStages][64] delta
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDl + kQStages * 64);
  uint64_t* kv_full = bars;
  uint64_t* st_full = kv_full + 1;           // [kQStages]
  uint64_t* st_empty = st_full + kQStages;   // [kQStages]
  uint64_t* sd_full = st_empty + kQStages;   // [2]
  uint64_t* pd_full = sd_full + 2;           // [2]
  uint64_t* buf_free = pd_full + 2;          // [2]
  uint64_t* acc_done = buf_free + 2;
  uint64_t* drain = acc_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr uint32_t kColDPT = 128, kColDV = 256, kColDK = 384;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x / p.Hkv;
  const int kvh = blockIdx.x - tile * p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int seq = p.ktiles[2 * tile];
  const int k0 = p.ktiles[2 * tile + 1];
  const int qbeg = p.cu_q[seq], nq = p.cu_q[seq + 1] - qbeg;
  const int kbeg = p.cu_k[seq], nk = p.cu_k[seq + 1] - kbeg;
  const int off = nk - nq;
  const int krows = min(128, nk - k0);
  // first query row that sees key k0 (bottom-right causal), rounded down to the sub-tile grid
  const int qstart = p.causal ? min(nq, max(0, k0 - off)) : 0;
  const int qs64 = (qstart / 64) * 64;
  const int nqs = (nq - qs64 + 63) / 64;
  const int steps = krows > 0 ? G * nqs : 0;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 128);  // two producer warps x (K, V)
    for (int s = 0; s < kQStages; ++s) {
      mbar_init(&st_full[s], 33);  // lane 0's expect-tx + 32 lanes' cp.async arrivals
      mbar_init(&st_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sd_full[b], 1);
      mbar_init(&pd_full[b], 8);
      mbar_init(&buf_free[b], 1);
    }
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&maps.q);
    tma_prefetch_desc(&maps.dO);
    tma_prefetch_desc(&maps.k);
    tma_prefetch_desc(&maps.v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int32_t* kidx = p.key_idx + kbeg + k0;

  if (warp == 0) {
    // ------------------------------------------------------------ Q_i / dO_i / lse / delta stream
    int last = -1;
    bool ok = true;
    for (int i = 0; i < steps && ok; ++i) {
      const int s = i % kQStages;
      if (!(ok = warp_wait(&st_empty[s], ((i / kQStages) & 1) ^ 1u, abort_flag, status, 960 + s))) break;
      const int hh = kvh * G + i / nqs;
      const int i0 = qs64 + (i % nqs) * 64;
      if (lane == 0) {
        mbar_arrive_expect_tx(&st_full[s], 2u * kTile64);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          tma_load_2d(sQ + s * kTile64 + half * kHalf64, &maps.q, &st_full[s], hh * kD + half * 64, qbeg + i0);
          tma_load_2d(sdO + s * kTile64 + half * kHalf64, &maps.dO, &st_full[s], hh * kD + half * 64, qbeg + i0);
        }
      }
      // lse / delta of the sub-tile's valid rows (the others stay stale: the mask never reads them)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = e * 32 + lane;
        if (i0 + c < nq) {
          const size_t gi = static_cast<size_t>(hh) * p.Tq + qbeg + i0 + c;
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(sL + s * 64 + c)), "l"(p.lse + gi)
                       : "memory");
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(sDl + s * 64 + c)), "l"(p.delta + gi)
                       : "memory");
        }
      }
      cp_async_arrive(&st_full[s]);
      last = i;
    }
    if (!ok) {
      asm volatile("cp.async.wait_all;" ::: "memory");
      if (lane == 0)
        for (int i = max(0, last - kQStages + 1); i <= last; ++i) drain_wait(&st_full[i % kQStages], (i / kQStages) & 1);
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ the key tile's K and V rows
    if (steps > 0) {
      const int rbase = (warp - 2) * 64;
      int ix[2], base;
      const bool contig = gather_rows(kidx, 0, rbase, krows, kidx[0], ix, base);
      load_gathered(sK, &maps.k, p.k + static_cast<size_t>(kvh) * kD, p.ldk, kv_full, rbase, kvh * kD, contig, base,
                    ix);
      load_gathered(sV, &maps.v, p.v + static_cast<size_t>(kvh) * kD, p.ldk, kv_full, rbase, kvh * kD, contig, base,
                    ix);
      // (the MMA warp waits for this phase before any read; on its timeout the copies still
      // land before the CTA exits: wait for them here)
      asm volatile("cp.async.wait_all;" ::: "memory");
      if (lane == 0) drain_wait(kv_full, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (event loop)
    if (lane == 0 && steps > 0) {
      constexpr uint32_t idesc_st = umma_idesc_f16(128, 64, false, false, true);
      constexpr uint32_t idesc_acc = umma_idesc_f16(128, kD, false, true, true);
      bool ok = mbar_wait(kv_full, 0, abort_flag, status, 970);
      const uint32_t kaddr = smem_u32(sK), vaddr = smem_u32(sV);
      int isd = 0, ivk = 0;
      bool issued = false;
      uint64_t t_last = globaltimer_ns();
      while (ok && ivk < steps) {
        bool progressed = false;
        // S^T(isd) = K Q^T, dP^T(isd) = V dO^T into buffer isd & 1
        if (isd < steps && isd - ivk < 2 && mbar_test(&st_full[isd % kQStages], (isd / kQStages) & 1) &&
            (isd < 2 || mbar_test(&buf_free[isd & 1], ((isd - 2) >> 1) & 1))) {
          tc_fence_after();
          fence_proxy_async_smem();  // cp.async-gathered K / V rows -> tensor-core reads
          const int b = isd & 1, s = isd % kQStages;
          const uint32_t qaddr = smem_u32(sQ + s * kTile64), doaddr = smem_u32(sdO + s * kTile64);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t ok_ = (kk >> 2) * kHalf + (kk & 3) * 32, oq = (kk >> 2) * kHalf64 + (kk & 3) * 32;
            umma_f16_ss(tmem + b * 64, umma_smem_desc(kaddr + ok_, 16, 1024), umma_smem_desc(qaddr + oq, 16, 1024),
                        idesc_st, kk > 0 ? 1u : 0u);
          }
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t ok_ = (kk >> 2) * kHalf + (kk & 3) * 32, oq = (kk >> 2) * kHalf64 + (kk & 3) * 32;
            umma_f16_ss(tmem + kColDPT + b * 64, umma_smem_desc(vaddr + ok_, 16, 1024),
                        umma_smem_desc(doaddr + oq, 16, 1024), idesc_st, kk > 0 ? 1u : 0u);
          }
          umma_commit(&sd_full[b]);
          ++isd;
          issued = progressed = true;
        }
        // dV += P^T dO_i, dK += dS^T Q_i
        if (ivk < isd && mbar_test(&pd_full[ivk & 1], (ivk >> 1) & 1)) {
          tc_fence_after();
          const int b = ivk & 1, s = ivk % kQStages;
          const uint32_t qaddr = smem_u32(sQ + s * kTile64), doaddr = smem_u32(sdO + s * kTile64);
          // A columns of query slice kk (16 queries): half kk / 2 at [32 (kk / 2), +16)
#pragma unroll
          for (int kk = 0; kk < 64 / 16; ++kk)
            umma_f16_ts(tmem + kColDV, tmem + b * 64 + (kk >> 1) * 32 + (kk & 1) * 8,
                        umma_smem_desc(doaddr + kk * 2048, kHalf64, 1024), idesc_acc, (ivk > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 64 / 16; ++kk)
            umma_f16_ts(tmem + kColDK, tmem + kColDPT + b * 64 + (kk >> 1) * 32 + (kk & 1) * 8,
                        umma_smem_desc(qaddr + kk * 2048, kHalf64, 1024), idesc_acc, (ivk > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&buf_free[b]);
          umma_commit(&st_empty[s]);
          ++ivk;
          issued = progressed = true;
        }
        if (progressed) {
          t_last = globaltimer_ns();
        } else if (*abort_flag) {
          ok = false;
        } else if (globaltimer_ns() - t_last > wait_budget_ns(status)) {
          *abort_flag = 1;
          record_error(status, kErrMbarTimeout, 980);
          ok = false;
        }
      }
      if (ok) umma_commit(acc_done);
      if (issued) {
        umma_commit(drain);
        drain_wait(drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ P^T, dS^T + epilogue (thread = key row)
    const int quarter = warp & 3;
    const int wh = (warp - 4) >> 2;             // query half of every sub-tile: [32 wh, 32 wh + 32)
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const bool kvalid = r < krows;
    const int qlo = p.causal ? k0 + r - off : 0;  // first query that sees this key
    const float sc = p.scale * kLog2e;
    bool ok = true;
    for (int i = 0; i < steps; ++i) {
      const int b = i & 1, s = i % kQStages;
      const int i0 = qs64 + (i % nqs) * 64 + wh * 32;
      // (the stage's lse / delta were written by cp.async: observe its barrier directly)
      if (!mbar_wait(&st_full[s], (i / kQStages) & 1, abort_flag, status, 990) ||
          !mbar_wait(&sd_full[b], (i >> 1) & 1, abort_flag, status, 991)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float* lse = sL + s * 64 + wh * 32;
      const float* dl = sDl + s * 64 + wh * 32;
      const uint32_t colS = b * 64 + wh * 32, colD = kColDPT + b * 64 + wh * 32;
      uint32_t sv[32], dv[32];
      tmem_ld_32x32b_x32(tmem + lane_addr + colS, sv);
      tmem_ld_32x32b_x32(tmem + lane_addr + colD, dv);
      tmem_wait_ld();
      uint32_t pp[16], dd[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int c = 2 * t;
        const int qi = i0 + c;
        const bool ok0 = kvalid && qi >= qlo && qi < nq;
        const bool ok1 = kvalid && qi + 1 >= qlo && qi + 1 < nq;
        const float p0 = ok0 ? exp2_approx(fmaf(__uint_as_float(sv[c]), sc, -lse[c] * kLog2e)) : 0.f;
        const float p1 = ok1 ? exp2_approx(fmaf(__uint_as_float(sv[c + 1]), sc, -lse[c + 1] * kLog2e)) : 0.f;
        pp[t] = pack_bf16x2(p0, p1);
        dd[t] = pack_bf16x2(ok0 ? p0 * (__uint_as_float(dv[c]) - dl[c]) : 0.f,
                            ok1 ? p1 * (__uint_as_float(dv[c + 1]) - dl[c + 1]) : 0.f);
      }
      // P^T / dS^T of this half -> the first 16 columns of its (already read) ranges
      tmem_st_32x32b_x16(tmem + lane_addr + colS, pp);
      tmem_st_32x32b_x16(tmem + lane_addr + colD, dd);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pd_full[b]);
    }
    // epilogue: half 0 adds dV, half 1 adds dK (x scale) into the gathered rows' accumulators
    if (ok && steps > 0 && mbar_wait(acc_done, 0, abort_flag, status, 995)) {
      tc_fence_after();
      const int64_t row = kvalid ? static_cast<int64_t>(kidx[r]) : 0;
      float* dst = (wh == 0 ? p.dv_acc : p.dk_acc) + row * p.ld_acc + static_cast<size_t>(kvh) * kD;
      const float mul = wh == 0 ? 1.f : p.scale;
      const uint32_t col = wh == 0 ? kColDV : kColDK;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + col + c * 32, v);
        tmem_wait_ld();
        if (kvalid) {
#pragma unroll
          for (int g = 0; g < 8; ++g)
            atomicAdd(reinterpret_cast<float4*>(dst + c * 32 + g * 4),
                      make_float4(__uint_as_float(v[g * 4]) * mul, __uint_as_float(v[g * 4 + 1]) * mul,
                                  __uint_as_float(v[g * 4 + 2]) * mul, __uint_as_float(v[g * 4 + 3]) * mul));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

int attn_bwd_dq_tc_smem_bytes() { return 6 * kTile + 1024 + 256; }
int attn_bwd_dkv_tc_smem_bytes() { return 2 * kTile + 2 * kQStages * kTile64 + 2 * kQStages * 64 * 4 + 1024 + 256; }

void attn_bwd_tc(const AttnBwdParams& p, const AttnBwdMaps& maps, int n_qtiles, int n_ktiles, int* status,
                 cudaStream_t st) {
  static SmemOptIn opt_dq, opt_dkv;
  opt_dq.ensure(attn_bwd_dq_tc_kernel, attn_bwd_dq_tc_smem_bytes());
  opt_dkv.ensure(attn_bwd_dkv_tc_kernel, attn_bwd_dkv_tc_smem_bytes());
  if (n_qtiles > 0)
    attn_bwd_dq_tc_kernel<<<n_qtiles * p.Hq, kThreads, attn_bwd_dq_tc_smem_bytes(), st>>>(maps, p, status);
  if (n_ktiles > 0)
    attn_bwd_dkv_tc_kernel<<<n_ktiles * p.Hkv, kThreads, attn_bwd_dkv_tc_smem_bytes(), st>>>(maps, p, status);
}

}  // namespace octo
