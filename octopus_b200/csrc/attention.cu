// Gathered-key attention for sm_100a.
//
// One formulation covers three users:
//   * prefix-tree training: each tree node attends to [mounted rows | ancestor path |
//     its own rows]; the key list of a node is a list of tree-row indices;
//   * paged prefill (page size 1): the key list of a request is its KV slot list;
//   * paged decode: one query row per request (split-K kernel below).
// The key rows are gathered straight from the K/V tensors by index (no index_select
// copy).  Causality is bottom-right aligned: query i of n_q sees key j of n_k iff
// j <= n_k - n_q + i, which is exact for "own rows last" key lists.
//
// Tensors: q [Tq, Hq, D] (row stride ldq), k/v [rows, Hkv, D] (row stride ldk),
// o [Tq, Hq, D] (row stride ldo), lse [Hq, Tq] fp32 natural-log normaliser.
// Sequences: cu_q[s]..cu_q[s+1] query rows, key_idx[cu_k[s]..cu_k[s+1]] key rows.
//
// Tensor-core path: mma.sync m16n8k16 bf16 with fp32 accumulation, K/V tiles gathered
// with cp.async into XOR-swizzled SMEM, online softmax in the exp2 domain.
#include <cuda_bf16.h>

#include "attention.h"
#include "common.cuh"

namespace octo {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `c` of row `r` in a [rows x D] bf16 tile, XOR swizzled.
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * (D * 2) + ((c ^ (r & 7)) << 4));
}

// Gather `ROWS` rows of D bf16 (one head) into a swizzled SMEM tile.  Row i comes from
// base + idx(i) * ld_elems; invalid rows are zero-filled.
template <int D, int ROWS, int NT>
__device__ __forceinline__ void load_tile_gather(uint32_t sbase, const bf16* base, int ld, const int32_t* idx,
                                                 int count, int tid) {
  constexpr int CH = D / 8;
#pragma unroll
  for (int i = tid; i < ROWS * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    const bool ok = r < count;
    const int64_t row = ok ? static_cast<int64_t>(idx[r]) : 0;
    cp_async16(sbase + swz<D>(r, c), base + row * ld + c * 8, ok);
  }
}
// Contiguous rows variant: row i = row0 + i.
template <int D, int ROWS, int NT>
__device__ __forceinline__ void load_tile_rows(uint32_t sbase, const bf16* base, int ld, int64_t row0, int count,
                                               int tid) {
  constexpr int CH = D / 8;
#pragma unroll
  for (int i = tid; i < ROWS * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    const bool ok = r < count;
    cp_async16(sbase + swz<D>(r, c), base + (row0 + (ok ? r : 0)) * ld + c * 8, ok);
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) { return pack_bf16x2(a, b); }

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ================================================================== forward
// CTA: 128 query rows of one sequence and one head (8 warps x 16 rows); K/V tiles of
// 64 keys double-buffered.
template <int D>
__global__ void __launch_bounds__(256, 1) attn_fwd_kernel(AttnParams p) {
  constexpr int BM = 128, BN = 64, NT = 256;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + BM * D * 2;
  const uint32_t sV0 = sK0 + 2 * BN * D * 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int seq = p.tiles[2 * blockIdx.x];
  const int q0 = p.tiles[2 * blockIdx.x + 1];
  const int h = blockIdx.y;
  const int kvh = h / (p.Hq / p.Hkv);
  const int qbeg = p.cu_q[seq], nq = p.cu_q[seq + 1] - qbeg;
  const int kbeg = p.cu_k[seq], nk = p.cu_k[seq + 1] - kbeg;
  const int off = nk - nq;
  const int mrows = min(BM, nq - q0);
  const int n_end = p.causal ? min(nk, q0 + mrows + off) : nk;

  const bf16* qb = p.q + static_cast<size_t>(h) * D;
  const bf16* kb = p.k + static_cast<size_t>(kvh) * D;
  const bf16* vb = p.v + static_cast<size_t>(kvh) * D;
  const int32_t* kidx = p.key_idx + kbeg;

  load_tile_rows<D, BM, NT>(sQ, qb, p.ldq, qbeg + q0, mrows, tid);
  cp_async_commit();
  const int n_tiles = (n_end + BN - 1) / BN;
  if (n_tiles > 0) {
    load_tile_gather<D, BN, NT>(sK0, kb, p.ldk, kidx, min(BN, n_end), tid);
    load_tile_gather<D, BN, NT>(sV0, vb, p.ldk, kidx, min(BN, n_end), tid);
  }
  cp_async_commit();

  // Q fragments: wait for the Q group only.
  cp_async_wait<1>();
  __syncthreads();
  uint32_t qf[D / 16][4];
  {
    const int r = warp * 16 + (lane & 15);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int c = kk * 2 + (lane >> 4);
      ldsm_x4(sQ + swz<D>(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const float sc = p.scale * kLog2e;
  const int g = lane >> 2, t4 = lane & 3;
  const int qi0 = q0 + warp * 16 + g;  // seq-relative query index of row g (row g+8 = qi0+8)

  for (int it = 0; it < n_tiles; ++it) {
    const int n0 = it * BN;
    const int buf = it & 1;
    if (it + 1 < n_tiles) {
      const int nn = n0 + BN;
      const uint32_t k_next = sK0 + (buf ^ 1) * BN * D * 2, v_next = sV0 + (buf ^ 1) * BN * D * 2;
      load_tile_gather<D, BN, NT>(k_next, kb, p.ldk, kidx + nn, min(BN, n_end - nn), tid);
      load_tile_gather<D, BN, NT>(v_next, vb, p.ldk, kidx + nn, min(BN, n_end - nn), tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t sK = sK0 + buf * BN * D * 2, sV = sV0 + buf * BN * D * 2;

    // S = Q K^T  (16 x 64 per warp)
    float s[BN / 8][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int jp = 0; jp < BN / 16; ++jp) {
        uint32_t b0, b1, b2, b3;
        const int r = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(sK + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(s[2 * jp], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma_bf16(s[2 * jp + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    }
    // mask + online softmax (exp2 domain)
    const bool need_mask = (n0 + BN > n_end) || (p.causal && n0 + BN - 1 > q0 + warp * 16 + off);
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int qi = qi0 + hr * 8;
      const int lim = p.causal ? min(n_end, qi + off + 1) : n_end;
      float mx = mrow[hr];
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float x = s[j][hr * 2 + e] * sc;
          if (need_mask) {
            const int kj = n0 + j * 8 + t4 * 2 + e;
            if (kj >= lim) x = -INFINITY;
          }
          s[j][hr * 2 + e] = x;
          mx = fmaxf(mx, x);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mref = (mx == -INFINITY) ? 0.f : mx;
      const float corr = exp2f(mrow[hr] - mref);
      mrow[hr] = mx;
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pv = exp2f(s[j][hr * 2 + e] - mref);
          s[j][hr * 2 + e] = pv;
          rs += pv;
        }
      }
      lrow[hr] = lrow[hr] * corr + rs;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][hr * 2] *= corr;
        o[i][hr * 2 + 1] *= corr;
      }
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      const uint32_t a0 = pack2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = dp * 2 + (lane >> 4);
        ldsm_x4_t(sV + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(o[2 * dp], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }

  // finalize
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float l = lrow[hr];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int qi = qi0 + hr * 8;
    if (qi - q0 < mrows) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* orow = p.o + static_cast<size_t>(qbeg + qi) * p.ldo + static_cast<size_t>(h) * D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        *reinterpret_cast<uint32_t*>(orow + i * 8 + t4 * 2) = pack2(o[i][hr * 2] * inv, o[i][hr * 2 + 1] * inv);
      }
      if (t4 == 0 && p.lse != nullptr) {
        p.lse[static_cast<size_t>(h) * p.Tq + qbeg + qi] = l > 0.f ? (mrow[hr] + log2f(l)) * kLn2 : -INFINITY;
      }
    }
  }
}

// ================================================================== backward
// delta[h, i] = sum_d dO[i, h, d] * O[i, h, d]
__global__ void attn_bwd_delta_kernel(const bf16* __restrict__ o, int ldo, const bf16* __restrict__ dO, int lddo,
                                      float* delta, int Tq, int Hq, int D) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= Tq * Hq) return;
  const int i = row / Hq, h = row % Hq;
  const bf16* a = o + static_cast<size_t>(i) * ldo + static_cast<size_t>(h) * D;
  const bf16* b = dO + static_cast<size_t>(i) * lddo + static_cast<size_t>(h) * D;
  float acc = 0.f;
  for (int c = lane * 2; c < D; c += 64) {
    const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(a + c));
    const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(b + c));
    acc += x.x * y.x + x.y * y.y;
  }
  acc = warp_sum(acc);
  if (lane == 0) delta[static_cast<size_t>(h) * Tq + i] = acc;
}

// dQ: CTA = 64 query rows (4 warps x 16) of one sequence/head, loop over key tiles.
template <int D>
__global__ void __launch_bounds__(128) attn_bwd_dq_kernel(AttnBwdParams p) {
  constexpr int BM = 64, BN = 64, NT = 128;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sdO = sQ + BM * D * 2;
  const uint32_t sK0 = sdO + BM * D * 2;
  const uint32_t sV0 = sK0 + 2 * BN * D * 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seq = p.tiles[2 * blockIdx.x];
  const int q0 = p.tiles[2 * blockIdx.x + 1];
  const int h = blockIdx.y;
  const int kvh = h / (p.Hq / p.Hkv);
  const int qbeg = p.cu_q[seq], nq = p.cu_q[seq + 1] - qbeg;
  const int kbeg = p.cu_k[seq], nk = p.cu_k[seq + 1] - kbeg;
  const int off = nk - nq;
  const int mrows = min(BM, nq - q0);
  const int n_end = p.causal ? min(nk, q0 + mrows + off) : nk;
  const bf16* kb = p.k + static_cast<size_t>(kvh) * D;
  const bf16* vb = p.v + static_cast<size_t>(kvh) * D;
  const int32_t* kidx = p.key_idx + kbeg;

  load_tile_rows<D, BM, NT>(sQ, p.q + static_cast<size_t>(h) * D, p.ldq, qbeg + q0, mrows, tid);
  load_tile_rows<D, BM, NT>(sdO, p.dO + static_cast<size_t>(h) * D, p.lddo, qbeg + q0, mrows, tid);
  cp_async_commit();
  const int n_tiles = (n_end + BN - 1) / BN;
  if (n_tiles > 0) {
    load_tile_gather<D, BN, NT>(sK0, kb, p.ldk, kidx, min(BN, n_end), tid);
    load_tile_gather<D, BN, NT>(sV0, vb, p.ldk, kidx, min(BN, n_end), tid);
  }
  cp_async_commit();

  const int g = lane >> 2, t4 = lane & 3;
  const int qi0 = q0 + warp * 16 + g;
  float lse2[2], dlt[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int qi = qi0 + hr * 8;
    const bool ok = qi < nq;
    lse2[hr] = ok ? p.lse[static_cast<size_t>(h) * p.Tq + qbeg + qi] * kLog2e : 0.f;
    dlt[hr] = ok ? p.delta[static_cast<size_t>(h) * p.Tq + qbeg + qi] : 0.f;
  }
  const float sc = p.scale * kLog2e;
  float dq[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;

  for (int it = 0; it < n_tiles; ++it) {
    const int n0 = it * BN, buf = it & 1;
    if (it + 1 < n_tiles) {
      const int nn = n0 + BN;
      load_tile_gather<D, BN, NT>(sK0 + (buf ^ 1) * BN * D * 2, kb, p.ldk, kidx + nn, min(BN, n_end - nn), tid);
      load_tile_gather<D, BN, NT>(sV0 + (buf ^ 1) * BN * D * 2, vb, p.ldk, kidx + nn, min(BN, n_end - nn), tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t sK = sK0 + buf * BN * D * 2, sV = sV0 + buf * BN * D * 2;
    float s[BN / 8][4], dp[BN / 8][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
      s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
      dp[j][0] = dp[j][1] = dp[j][2] = dp[j][3] = 0.f;
    }
    const int ar = warp * 16 + (lane & 15);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a0, a1, a2, a3, d0, d1, d2, d3;
      const int ac = kk * 2 + (lane >> 4);
      ldsm_x4(sQ + swz<D>(ar, ac), a0, a1, a2, a3);
      ldsm_x4(sdO + swz<D>(ar, ac), d0, d1, d2, d3);
#pragma unroll
      for (int jp = 0; jp < BN / 16; ++jp) {
        uint32_t b0, b1, b2, b3;
        const int r = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(sK + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(s[2 * jp], a0, a1, a2, a3, b0, b1);
        mma_bf16(s[2 * jp + 1], a0, a1, a2, a3, b2, b3);
        ldsm_x4(sV + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(dp[2 * jp], d0, d1, d2, d3, b0, b1);
        mma_bf16(dp[2 * jp + 1], d0, d1, d2, d3, b2, b3);
      }
    }
    // dS = P * (dP - delta)   (P recomputed from lse)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int qi = qi0 + hr * 8;
      const int lim = p.causal ? min(n_end, qi + off + 1) : n_end;
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kj = n0 + j * 8 + t4 * 2 + e;
          float pv = exp2f(s[j][hr * 2 + e] * sc - lse2[hr]);
          if (kj >= lim || qi >= nq) pv = 0.f;
          s[j][hr * 2 + e] = pv * (dp[j][hr * 2 + e] - dlt[hr]);
        }
      }
    }
    // dQ += dS K
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      const uint32_t a0 = pack2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dpi = 0; dpi < D / 16; ++dpi) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = dpi * 2 + (lane >> 4);
        ldsm_x4_t(sK + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(dq[2 * dpi], a0, a1, a2, a3, b0, b1);
        mma_bf16(dq[2 * dpi + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int qi = qi0 + hr * 8;
    if (qi < nq && qi - q0 < mrows) {
      bf16* row = p.dq + static_cast<size_t>(qbeg + qi) * p.lddq + static_cast<size_t>(h) * D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i)
        *reinterpret_cast<uint32_t*>(row + i * 8 + t4 * 2) =
            pack2(dq[i][hr * 2] * p.scale, dq[i][hr * 2 + 1] * p.scale);
    }
  }
}

// dK, dV: CTA = 64 keys of one sequence's key list (4 warps x 16 keys) and one kv head;
// loops over the q heads of the GQA group and 32-row query tiles, then adds its
// partial sums into the fp32 dK/dV accumulators of the gathered rows (rows are shared
// between sequences, e.g. a tree prefix seen by every descendant).
template <int D>
__global__ void __launch_bounds__(128) attn_bwd_dkv_kernel(AttnBwdParams p) {
  constexpr int BK = 64, BQ = 32, NT = 128;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BK * D * 2;
  const uint32_t sQ0 = sV + BK * D * 2;        // 2 stages
  const uint32_t sdO0 = sQ0 + 2 * BQ * D * 2;  // 2 stages
  float* s_lse = reinterpret_cast<float*>(smem + (2 * BK + 4 * BQ) * D * 2);  // [2][BQ]
  float* s_dlt = s_lse + 2 * BQ;                                              // [2][BQ]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seq = p.ktiles[2 * blockIdx.x];
  const int k0 = p.ktiles[2 * blockIdx.x + 1];
  const int kvh = blockIdx.y;
  const int G = p.Hq / p.Hkv;
  const int qbeg = p.cu_q[seq], nq = p.cu_q[seq + 1] - qbeg;
  const int kbeg = p.cu_k[seq], nk = p.cu_k[seq + 1] - kbeg;
  const int off = nk - nq;
  const int krows = min(BK, nk - k0);
  const int32_t* kidx = p.key_idx + kbeg + k0;

  load_tile_gather<D, BK, NT>(sK, p.k + static_cast<size_t>(kvh) * D, p.ldk, kidx, krows, tid);
  load_tile_gather<D, BK, NT>(sV, p.v + static_cast<size_t>(kvh) * D, p.ldk, kidx, krows, tid);
  cp_async_commit();

  // first query row that can see key k0 (causal): i >= k0 - off
  const int qstart = p.causal ? max(0, k0 - off) : 0;
  const int qtiles = qstart < nq ? (nq - qstart + BQ - 1) / BQ : 0;
  const int steps = qtiles * G;
  const float sc = p.scale * kLog2e;
  const int g = lane >> 2, t4 = lane & 3;

  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }

  auto issue = [&](int step, int buf) {
    const int hh = kvh * G + step / qtiles;
    const int qt = step % qtiles;
    const int i0 = qstart + qt * BQ;
    const int cnt = min(BQ, nq - i0);
    load_tile_rows<D, BQ, NT>(sQ0 + buf * BQ * D * 2, p.q + static_cast<size_t>(hh) * D, p.ldq, qbeg + i0, cnt,
                              tid);
    load_tile_rows<D, BQ, NT>(sdO0 + buf * BQ * D * 2, p.dO + static_cast<size_t>(hh) * D, p.lddo, qbeg + i0, cnt,
                              tid);
  };
  if (steps > 0) issue(0, 0);
  cp_async_commit();

  for (int step = 0; step < steps; ++step) {
    const int buf = step & 1;
    const int hh = kvh * G + step / qtiles;
    const int i0 = qstart + (step % qtiles) * BQ;
    if (tid < BQ) {
      const int qi = i0 + tid;
      const bool ok = qi < nq;
      s_lse[buf * BQ + tid] = ok ? p.lse[static_cast<size_t>(hh) * p.Tq + qbeg + qi] * kLog2e : INFINITY;
      s_dlt[buf * BQ + tid] = ok ? p.delta[static_cast<size_t>(hh) * p.Tq + qbeg + qi] : 0.f;
    }
    if (step + 1 < steps) issue(step + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t sQ = sQ0 + buf * BQ * D * 2, sdO = sdO0 + buf * BQ * D * 2;

    // S^T = K Q^T and dP^T = V dO^T  (16 keys x 32 queries per warp)
    float st[BQ / 8][4], dpt[BQ / 8][4];
#pragma unroll
    for (int j = 0; j < BQ / 8; ++j) {
      st[j][0] = st[j][1] = st[j][2] = st[j][3] = 0.f;
      dpt[j][0] = dpt[j][1] = dpt[j][2] = dpt[j][3] = 0.f;
    }
    const int ar = warp * 16 + (lane & 15);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a0, a1, a2, a3, v0, v1, v2, v3;
      const int ac = kk * 2 + (lane >> 4);
      ldsm_x4(sK + swz<D>(ar, ac), a0, a1, a2, a3);
      ldsm_x4(sV + swz<D>(ar, ac), v0, v1, v2, v3);
#pragma unroll
      for (int jp = 0; jp < BQ / 16; ++jp) {
        uint32_t b0, b1, b2, b3;
        const int r = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(sQ + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(st[2 * jp], a0, a1, a2, a3, b0, b1);
        mma_bf16(st[2 * jp + 1], a0, a1, a2, a3, b2, b3);
        ldsm_x4(sdO + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(dpt[2 * jp], v0, v1, v2, v3, b0, b1);
        mma_bf16(dpt[2 * jp + 1], v0, v1, v2, v3, b2, b3);
      }
    }
    // P^T and dS^T; rows = keys (k0 + warp*16 + g (+8)), cols = queries
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int kj = k0 + warp * 16 + g + hr * 8;
#pragma unroll
      for (int j = 0; j < BQ / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int qc = j * 8 + t4 * 2 + e;
          const int qi = i0 + qc;
          float pv = exp2f(st[j][hr * 2 + e] * sc - s_lse[buf * BQ + qc]);
          const bool ok = kj < nk && qi < nq && (!p.causal || kj <= qi + off);
          if (!ok) pv = 0.f;
          st[j][hr * 2 + e] = pv;
          dpt[j][hr * 2 + e] = pv * (dpt[j][hr * 2 + e] - s_dlt[buf * BQ + qc]);
        }
      }
    }
    // dV += P^T dO ; dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
      const uint32_t p0 = pack2(st[2 * kk][0], st[2 * kk][1]);
      const uint32_t p1 = pack2(st[2 * kk][2], st[2 * kk][3]);
      const uint32_t p2 = pack2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      const uint32_t p3 = pack2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
      const uint32_t d0 = pack2(dpt[2 * kk][0], dpt[2 * kk][1]);
      const uint32_t d1 = pack2(dpt[2 * kk][2], dpt[2 * kk][3]);
      const uint32_t d2 = pack2(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
      const uint32_t d3 = pack2(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
#pragma unroll
      for (int dpi = 0; dpi < D / 16; ++dpi) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = dpi * 2 + (lane >> 4);
        ldsm_x4_t(sdO + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(dv[2 * dpi], p0, p1, p2, p3, b0, b1);
        mma_bf16(dv[2 * dpi + 1], p0, p1, p2, p3, b2, b3);
        ldsm_x4_t(sQ + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(dk[2 * dpi], d0, d1, d2, d3, b0, b1);
        mma_bf16(dk[2 * dpi + 1], d0, d1, d2, d3, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  // scatter-add into fp32 accumulators of the gathered rows
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int kr = warp * 16 + g + hr * 8;
    if (kr < krows) {
      const int64_t row = kidx[kr];
      float* dkr = p.dk_acc + row * p.ld_acc + static_cast<size_t>(kvh) * D;
      float* dvr = p.dv_acc + row * p.ld_acc + static_cast<size_t>(kvh) * D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        atomicAdd(dkr + i * 8 + t4 * 2, dk[i][hr * 2] * p.scale);
        atomicAdd(dkr + i * 8 + t4 * 2 + 1, dk[i][hr * 2 + 1] * p.scale);
        atomicAdd(dvr + i * 8 + t4 * 2, dv[i][hr * 2]);
        atomicAdd(dvr + i * 8 + t4 * 2 + 1, dv[i][hr * 2 + 1]);
      }
    }
  }
}

// ================================================================== paged decode
// One query row per request; GQA group rows packed into the 16-row MMA tile.
// CTA = (request, kv head, split); 4 warps each walk 32-key tiles of the split range.
template <int D>
__global__ void __launch_bounds__(128) attn_decode_kernel(DecodeParams p) {
  constexpr int BN = 32, NW = 4;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int G = p.Hq / p.Hkv;
  const int kbeg = p.kv_start[b], nk = p.kv_len[b];
  const int per = ((nk + p.num_splits - 1) / p.num_splits + BN - 1) / BN * BN;
  const int s_beg = split * per, s_end = min(nk, s_beg + per);
  // per-warp double-buffered K/V tiles
  const uint32_t wbase = smem_u32(smem) + warp * (2 * 2 * BN * D * 2);
  float* red = reinterpret_cast<float*>(smem);  // [NW][16][D+2], used after the key loop
  const bf16* kb = p.k_cache + static_cast<size_t>(kvh) * D;
  const bf16* vb = p.v_cache + static_cast<size_t>(kvh) * D;
  const int32_t* kidx = p.kv_indices + kbeg;

  // Q fragments straight from global (rows = heads of the group, zero padded to 16)
  const int g = lane >> 2, t4 = lane & 3;
  uint32_t qf[D / 16][4];
  {
    const bf16* qrow_g = p.q + static_cast<size_t>(b) * p.ldq + static_cast<size_t>(kvh * G + g) * D;
    const bf16* qrow_g8 = p.q + static_cast<size_t>(b) * p.ldq + static_cast<size_t>(kvh * G + g + 8) * D;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int c = kk * 16 + t4 * 2;
      qf[kk][0] = g < G ? *reinterpret_cast<const uint32_t*>(qrow_g + c) : 0u;
      qf[kk][1] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qrow_g8 + c) : 0u;
      qf[kk][2] = g < G ? *reinterpret_cast<const uint32_t*>(qrow_g + c + 8) : 0u;
      qf[kk][3] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qrow_g8 + c + 8) : 0u;
    }
  }
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const float sc = p.scale * kLog2e;

  // warp-private tile sequence: tiles w, w+NW, ...
  const int ntiles = s_end > s_beg ? (s_end - s_beg + BN - 1) / BN : 0;
  auto issue = [&](int tix, int buf) {
    const int n0 = s_beg + tix * BN;
    const int cnt = min(BN, s_end - n0);
    const uint32_t sk = wbase + buf * 2 * BN * D * 2, sv = sk + BN * D * 2;
    constexpr int CH = D / 8;
#pragma unroll
    for (int i = lane; i < BN * CH; i += 32) {
      const int r = i / CH, c = i % CH;
      const bool ok = r < cnt;
      const int64_t row = ok ? static_cast<int64_t>(kidx[n0 + r]) : 0;
      cp_async16(sk + swz<D>(r, c), kb + row * p.ldk + c * 8, ok);
      cp_async16(sv + swz<D>(r, c), vb + row * p.ldk + c * 8, ok);
    }
  };
  int it = 0;
  if (warp < ntiles) issue(warp, 0);
  cp_async_commit();
  for (int tix = warp; tix < ntiles; tix += NW, ++it) {
    const int buf = it & 1;
    if (tix + NW < ntiles) issue(tix + NW, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    const uint32_t sk = wbase + buf * 2 * BN * D * 2, sv = sk + BN * D * 2;
    const int n0 = s_beg + tix * BN;
    float s[BN / 8][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int jp = 0; jp < BN / 16; ++jp) {
        uint32_t b0, b1, b2, b3;
        const int r = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(sk + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(s[2 * jp], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma_bf16(s[2 * jp + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = mrow[hr];
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kj = n0 + j * 8 + t4 * 2 + e;
          float x = s[j][hr * 2 + e] * sc;
          if (kj >= s_end) x = -INFINITY;
          s[j][hr * 2 + e] = x;
          mx = fmaxf(mx, x);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mref = (mx == -INFINITY) ? 0.f : mx;
      const float corr = exp2f(mrow[hr] - mref);
      mrow[hr] = mx;
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pv = exp2f(s[j][hr * 2 + e] - mref);
          s[j][hr * 2 + e] = pv;
          rs += pv;
        }
      }
      lrow[hr] = lrow[hr] * corr + rs;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][hr * 2] *= corr;
        o[i][hr * 2 + 1] *= corr;
      }
    }
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      const uint32_t a0 = pack2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = dp * 2 + (lane >> 4);
        ldsm_x4_t(sv + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(o[2 * dp], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  // combine the 4 warps: (m, l, o) per row via SMEM (reusing the tile buffers)
  constexpr int RS = D + 2;
  __syncthreads();
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float l = lrow[hr];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int r = g + hr * 8;
    float* rw = red + (warp * 16 + r) * RS;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      rw[i * 8 + t4 * 2] = o[i][hr * 2];
      rw[i * 8 + t4 * 2 + 1] = o[i][hr * 2 + 1];
    }
    if (t4 == 0) {
      rw[D] = mrow[hr];
      rw[D + 1] = l;
    }
  }
  __syncthreads();
  // thread layout for the combine: rows r < G, columns spread over the CTA
  for (int idx = tid; idx < G * D; idx += blockDim.x) {
    const int r = idx / D, c = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, red[(w * 16 + r) * RS + D]);
    float L = 0.f, acc = 0.f;
    const float mref = M == -INFINITY ? 0.f : M;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float* rw = red + (w * 16 + r) * RS;
      const float f = exp2f(rw[D] - mref);
      L += rw[D + 1] * f;
      acc += rw[c] * f;
    }
    const int hq = kvh * G + r;
    if (p.num_splits == 1) {
      bf16* orow = p.o + static_cast<size_t>(b) * p.ldo + static_cast<size_t>(hq) * D;
      orow[c] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
    } else {
      const size_t base = (static_cast<size_t>(b) * p.Hq + hq) * p.num_splits + split;
      p.part_o[base * D + c] = L > 0.f ? acc / L : 0.f;
      if (c == 0) p.part_lse[base] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
}

__global__ void attn_decode_combine_kernel(DecodeParams p, int D) {
  const int b = blockIdx.x, hq = blockIdx.y;
  const size_t base = (static_cast<size_t>(b) * p.Hq + hq) * p.num_splits;
  float M = -INFINITY;
  for (int s = 0; s < p.num_splits; ++s) M = fmaxf(M, p.part_lse[base + s]);
  const float mref = M == -INFINITY ? 0.f : M;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float L = 0.f, acc = 0.f;
    for (int s = 0; s < p.num_splits; ++s) {
      const float w = exp2f(p.part_lse[base + s] - mref);
      L += w;
      acc += w * p.part_o[(base + s) * D + c];
    }
    p.o[static_cast<size_t>(b) * p.ldo + static_cast<size_t>(hq) * D + c] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
  }
}

// ================================================================== host launchers
template <int D>
static int fwd_smem() {
  return 128 * D * 2 + 2 * 2 * 64 * D * 2;
}
template <int D>
static int dq_smem() {
  return 2 * 64 * D * 2 + 2 * 2 * 64 * D * 2;
}
template <int D>
static int dkv_smem() {
  return (2 * 64 + 4 * 32) * D * 2 + 4 * 32 * sizeof(float);
}
template <int D>
static int dec_smem() {
  const int tiles = 4 * 2 * 2 * 32 * D * 2;
  const int red = 4 * 16 * (D + 2) * static_cast<int>(sizeof(float));
  return tiles > red ? tiles : red;
}

template <int D>
static void fwd_impl(const AttnParams& p, int n_tiles, cudaStream_t st) {
  static SmemOptIn opt;
  opt.ensure(attn_fwd_kernel<D>, fwd_smem<D>());
  attn_fwd_kernel<D><<<dim3(n_tiles, p.Hq), 256, fwd_smem<D>(), st>>>(p);
}

void attn_fwd(const AttnParams& p, int n_tiles, int D, cudaStream_t st) {
  if (n_tiles == 0) return;
  if (D == 128) fwd_impl<128>(p, n_tiles, st);
  else fwd_impl<64>(p, n_tiles, st);
}

template <int D>
static void bwd_impl(const AttnBwdParams& p, int n_qtiles, int n_ktiles, cudaStream_t st) {
  static SmemOptIn opt_dq, opt_dkv;
  opt_dq.ensure(attn_bwd_dq_kernel<D>, dq_smem<D>());
  opt_dkv.ensure(attn_bwd_dkv_kernel<D>, dkv_smem<D>());
  if (n_qtiles > 0) attn_bwd_dq_kernel<D><<<dim3(n_qtiles, p.Hq), 128, dq_smem<D>(), st>>>(p);
  if (n_ktiles > 0) attn_bwd_dkv_kernel<D><<<dim3(n_ktiles, p.Hkv), 128, dkv_smem<D>(), st>>>(p);
}

void attn_bwd_delta(const bf16* o, int ldo, const bf16* dO, int lddo, float* delta, int Tq, int Hq, int D,
                    cudaStream_t st) {
  if (Tq == 0) return;
  const int rows = Tq * Hq;
  attn_bwd_delta_kernel<<<(rows + 7) / 8, 256, 0, st>>>(o, ldo, dO, lddo, delta, Tq, Hq, D);
}

void attn_bwd(const AttnBwdParams& p, int n_qtiles, int n_ktiles, int D, cudaStream_t st) {
  if (D == 128) bwd_impl<128>(p, n_qtiles, n_ktiles, st);
  else bwd_impl<64>(p, n_qtiles, n_ktiles, st);
}

// Launches through cudaLaunchKernelEx so that the returned code is this call's own
// (an error left pending by unrelated earlier work is neither reported nor cleared).
template <int D>
static cudaError_t dec_impl(const DecodeParams& p, int B, cudaStream_t st) {
  static SmemOptIn opt;
  cudaError_t e = opt.ensure(attn_decode_kernel<D>, dec_smem<D>());
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(B, p.Hkv, p.num_splits);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = dec_smem<D>();
  cfg.stream = st;
  e = cudaLaunchKernelEx(&cfg, attn_decode_kernel<D>, p);
  if (e != cudaSuccess || p.num_splits <= 1) return e;
  cudaLaunchConfig_t cc{};
  cc.gridDim = dim3(B, p.Hq);
  cc.blockDim = dim3(128);
  cc.stream = st;
  return cudaLaunchKernelEx(&cc, attn_decode_combine_kernel, p, D);
}

cudaError_t attn_decode(const DecodeParams& p, int B, int D, cudaStream_t st) {
  if (B == 0) return cudaSuccess;
  return D == 128 ? dec_impl<128>(p, B, st) : dec_impl<64>(p, B, st);
}

}  // namespace octo
