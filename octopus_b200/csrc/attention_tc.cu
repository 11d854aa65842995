// Gathered-key attention forward on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same contract as attn_fwd in attention.cu (tree nodes / paged prefill: query rows of
// a sequence attend to a gathered key list, bottom-right causal, GQA), head_dim 128.
//
// CTA = 128 query rows of one sequence and one head; 224 threads:
//   warps 0-1   producers: cp.async gathers of Q (once) and of 128-key K/V tiles into a
//               2-stage SMEM ring (128-byte swizzled K-major layout that the UMMA
//               descriptors read directly), 64 rows per warp; completion via
//               cp.async.mbarrier.arrive
//   warp 2      TMEM owner and single-thread MMA issuer, event driven: S_{j+1} is issued
//               as soon as K_{j+1} has landed and its S buffer is free, P_j V_j as soon as
//               the softmax has written P_j:
//                 S_j = Q K_j^T         tcgen05.mma kind::f16, A/B from SMEM, fp32 in TMEM
//                 O  += P_{j-1} V_{j-1}  tcgen05.mma with A = P read from TMEM (bf16),
//                                        B = V from SMEM (MN-major)
//   warps 3..6  softmax: thread = query row (TMEM lane), S row loaded with tcgen05.ld,
//               online softmax in the exp2 domain with lazy rescaling (O is rescaled in
//               TMEM only when the running max grows by more than 2^8), P written back
//               to TMEM as packed bf16; epilogue O / l -> bf16 rows + lse.
// TMEM columns: S double buffer [0,256), P [256,320), O [384,512).
// All mbarrier waits are bounded (common.cuh); on timeout the CTA records an error,
// drains its MMAs and frees TMEM.
#include <cuda_bf16.h>

#include "attention.h"
#include "common.cuh"

namespace octo {

namespace {

constexpr int kBM = 128, kBN = 128, kD = 128;
constexpr int kHalf = 128 * 128;            // bytes of one 64-column half of a 128-row tile
constexpr int kTileBytes = 2 * kHalf;       // 32 KB: a 128 x 128 bf16 tile
constexpr int kStages = 2;
constexpr uint32_t kColS = 0, kColP = 256, kColO = 384;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;   // log2 units

__device__ __forceinline__ uint32_t toff(int r, int c) {
  // row r, 16-byte chunk c (0..15) of a 128 x 128 bf16 tile made of two SW128 halves
  return static_cast<uint32_t>((c >> 3) * kHalf + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Trace slots (the last CTA of head 0 only, when p.trace != nullptr): [role * 64 + tile] = globaltimer.
__device__ __forceinline__ void trace_at(const AttnParams& p, int role, int idx) {
  if (p.trace != nullptr && blockIdx.x == gridDim.x - 1 && blockIdx.y == 0 && idx < 64) p.trace[role * 64 + idx] = globaltimer_ns();
}

}  // namespace

constexpr int kProducers = 2;  // 64 rows each (register budget: 7 warps keep 255 regs/thread)
constexpr int kThreads = (kProducers + 1 + 4) * 32;

__global__ void __launch_bounds__(kThreads, 1) attn_fwd_tc_kernel(AttnParams p, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kTileBytes;                   // kStages tiles
  uint8_t* sV = sK + kStages * kTileBytes;           // kStages tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kStages * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                      // [kStages]
  uint64_t* kv_empty = kv_full + kStages;            // [kStages]
  uint64_t* s_full = kv_empty + kStages;             // [2]
  uint64_t* s_empty = s_full + 2;                    // [2]
  uint64_t* p_full = s_empty + 2;
  uint64_t* o_done = p_full + 1;
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = p.tiles[2 * blockIdx.x];
  const int q0 = p.tiles[2 * blockIdx.x + 1];
  const int h = blockIdx.y;
  const int kvh = h / (p.Hq / p.Hkv);
  const int qbeg = p.cu_q[seq], nq = p.cu_q[seq + 1] - qbeg;
  const int kbeg = p.cu_k[seq], nk = p.cu_k[seq + 1] - kbeg;
  const int off = nk - nq;
  const int mrows = min(kBM, nq - q0);
  const int n_end = p.causal ? min(nk, q0 + mrows + off) : nk;
  const int n_tiles = (n_end + kBN - 1) / kBN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 32 * kProducers);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 32 * kProducers);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProducers) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) trace_at(p, 9, 0);

  if (warp < kProducers) {
    // ------------------------------------------------------------ producers (32 rows each)
    const __nv_bfloat16* qb = p.q + static_cast<size_t>(h) * kD;
    const __nv_bfloat16* kb = p.k + static_cast<size_t>(kvh) * kD;
    const __nv_bfloat16* vb = p.v + static_cast<size_t>(kvh) * kD;
    const int32_t* kidx = p.key_idx + kbeg;
    const int cl = lane & 15;      // 16 lanes per row: coalesced 256-byte row reads
    constexpr int kRows = kBM / kProducers;
    const int rbase = warp * kRows;  // this warp's rows of every tile
    {
      const uint32_t base = smem_u32(sQ);
#pragma unroll
      for (int i = 0; i < kRows / 2; ++i) {
        const int r = rbase + 2 * i + (lane >> 4);
        const __nv_bfloat16* src = qb + static_cast<size_t>(qbeg + q0 + (r < mrows ? r : 0)) * p.ldq;
        cp_async16(base + toff(r, cl), src + cl * 8);
      }
      cp_async_arrive(q_full);
    }
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    const int32_t first = nk > 0 ? kidx[0] : 0;
    // this warp's slot indices: one coalesced load per 32 rows, handed out by shuffle;
    // rows past the key list read a valid row (the softmax masks them).  Loaded one tile
    // ahead so their latency hides behind the wait and the current tile's copies.
    int nx[kRows / 32];
#pragma unroll
    for (int q = 0; q < kRows / 32; ++q) {
      const int kk = rbase + q * 32 + lane;
      nx[q] = kk < n_end ? static_cast<int>(kidx[kk]) : first;
    }
    for (int j = 0; j < n_tiles && ok; ++j) {
      int ix[kRows / 32];
#pragma unroll
      for (int q = 0; q < kRows / 32; ++q) ix[q] = nx[q];
      if (j + 1 < n_tiles) {
#pragma unroll
        for (int q = 0; q < kRows / 32; ++q) {
          const int kk = (j + 1) * kBN + rbase + q * 32 + lane;
          nx[q] = kk < n_end ? static_cast<int>(kidx[kk]) : first;
        }
      }
      if (lane == 0) ok = mbar_wait(&kv_empty[stage], phase ^ 1u, abort_flag, status, 500 + stage);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      if (warp == 0 && lane == 0) trace_at(p, 0, j);
      const uint32_t kbase = smem_u32(sK + stage * kTileBytes);
      const uint32_t vbase = smem_u32(sV + stage * kTileBytes);
#pragma unroll
      for (int i = 0; i < kRows / 2; ++i) {
        const int rl = 2 * i + (lane >> 4);
        const int64_t row = static_cast<int64_t>(__shfl_sync(0xffffffffu, ix[rl >> 5], rl & 31));
        const int r = rbase + rl;
        cp_async16(kbase + toff(r, cl), kb + row * p.ldk + cl * 8);
        cp_async16(vbase + toff(r, cl), vb + row * p.ldk + cl * 8);
      }
      cp_async_arrive(&kv_full[stage]);
      if (warp == 0 && lane == 0) trace_at(p, 1, j);
      if (++stage == kStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
  } else if (warp == kProducers) {
    // ------------------------------------------------------------ MMA issuer (event loop)
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(kBM, kBN, false, false, true);
      constexpr uint32_t idesc_o = umma_idesc_f16(kBM, kD, false, true, true);
      bool ok = mbar_wait(q_full, 0, abort_flag, status, 600);
      fence_proxy_async_smem();  // cp.async (generic proxy) writes -> tensor-core reads
      const uint32_t qaddr = smem_u32(sQ);
      int js = 0, jp = 0;        // next tile whose S / P.V to issue
      bool issued = false;
      const uint64_t t_start = globaltimer_ns();
      uint64_t t_last = t_start;
      while (ok && jp < n_tiles) {
        bool progressed = false;
        if (js < n_tiles && js - jp < kStages) {
          const int st = js % kStages;
          const uint32_t ph = static_cast<uint32_t>((js / kStages) & 1);
          const int b = js & 1;
          if (mbar_test(&kv_full[st], ph) && mbar_test(&s_empty[b], ((js >> 1) & 1) ^ 1u)) {
            tc_fence_after();
            fence_proxy_async_smem();
            trace_at(p, 2, js);
            const uint32_t kaddr = smem_u32(sK + st * kTileBytes);
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t o16 = (kk >> 2) * kHalf + (kk & 3) * 32;
              const uint64_t ad = umma_smem_desc(qaddr + o16, 16, 1024);
              const uint64_t bd = umma_smem_desc(kaddr + o16, 16, 1024);
              umma_f16_ss(tmem + kColS + b * 128, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[b]);
            trace_at(p, 3, js);
            issued = true;
            ++js;
            progressed = true;
          }
        }
        if (jp < js && mbar_test(p_full, jp & 1)) {
          tc_fence_after();
          trace_at(p, 4, jp);
          const int st = jp % kStages;
          const uint32_t vaddr = smem_u32(sV + st * kTileBytes);
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint64_t bd = umma_smem_desc(vaddr + kk * 2048, kHalf, 1024);
            umma_f16_ts(tmem + kColO, tmem + kColP + kk * 8, bd, idesc_o, (jp > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(o_done);
          umma_commit(&kv_empty[st]);
          ++jp;
          progressed = true;
        }
        if (progressed) {
          t_last = globaltimer_ns();
        } else if (*abort_flag) {
          ok = false;
        } else if (globaltimer_ns() - t_last > wait_budget_ns(status)) {
          *abort_flag = 1;
          record_error(status, kErrMbarTimeout, 610);
          ok = false;
        }
      }
      if (issued) {
        umma_commit(drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (globaltimer_ns() - t0 > OCTO_WAIT_NS) break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (128 threads)
    const int quarter = warp & 3;               // warps 3..6 -> TMEM lane quarters 3, 0, 1, 2
    const int r = quarter * 32 + lane;          // TMEM lane = query row in the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int qi = q0 + r;                      // sequence-relative query index
    const int lim = p.causal ? min(n_end, qi + off + 1) : n_end;
    const float sc = p.scale * kLog2e;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int b = j & 1;
      if (!mbar_wait(&s_full[b], (j >> 1) & 1, abort_flag, status, 650 + b)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (threadIdx.x == (kProducers + 1) * 32) trace_at(p, 5, j);
      float s[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + kColS + b * 128 + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(v[i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[b]);
      if (threadIdx.x == (kProducers + 1) * 32) trace_at(p, 6, j);
      const int kbase = j * kBN;
      float mt = -INFINITY;
#pragma unroll
      for (int i = 0; i < kBN; ++i) {
        const float x = (kbase + i < lim) ? s[i] * sc : -INFINITY;
        s[i] = x;
        mt = fmaxf(mt, x);
      }
      float alpha = 1.f;
      if (j == 0) {
        m = mt;
      } else if (mt > m + kRescaleThreshold) {
        alpha = exp2f(m - mt);
        m = mt;
      }
      const float mref = m == -INFINITY ? 0.f : m;
      float rs = 0.f;
      uint32_t pk[kBN / 2];
#pragma unroll
      for (int i = 0; i < kBN / 2; ++i) {
        const float a = exp2_approx(s[2 * i] - mref), bb = exp2_approx(s[2 * i + 1] - mref);
        rs += a + bb;
        pk[i] = pack_bf16x2(a, bb);
      }
      l = l * alpha + rs;
      if (j > 0) {
        // the previous P.V must be complete before P is overwritten or O is rescaled
        if (!mbar_wait(o_done, (j - 1) & 1, abort_flag, status, 660)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (threadIdx.x == (kProducers + 1) * 32) trace_at(p, 7, j);
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < kD / 32; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + lane_addr + kColO + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
            tmem_st_32x32b_x32(tmem + lane_addr + kColO + c * 32, v);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = pk[c * 32 + i];
        tmem_st_32x32b_x32(tmem + lane_addr + kColP + c * 32, v);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (threadIdx.x == (kProducers + 1) * 32) trace_at(p, 8, j);
    }
    // epilogue: O / l
    if (ok && n_tiles > 0 && mbar_wait(o_done, (n_tiles - 1) & 1, abort_flag, status, 670)) {
      tc_fence_after();
      const bool write = r < mrows;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + static_cast<size_t>(qbeg + q0 + (write ? r : 0)) * p.ldo + static_cast<size_t>(h) * kD;
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + kColO + c * 32, v);
        tmem_wait_ld();
        if (write) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(v[g * 8 + 0]) * inv, __uint_as_float(v[g * 8 + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(v[g * 8 + 2]) * inv, __uint_as_float(v[g * 8 + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(v[g * 8 + 4]) * inv, __uint_as_float(v[g * 8 + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(v[g * 8 + 6]) * inv, __uint_as_float(v[g * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + g * 8) = u;
          }
        }
      }
      if (write && p.lse != nullptr)
        p.lse[static_cast<size_t>(h) * p.Tq + qbeg + q0 + r] = l > 0.f ? (m + log2f(l)) * kLn2 : -INFINITY;
    } else if (n_tiles == 0 && r < mrows) {
      __nv_bfloat16* orow = p.o + static_cast<size_t>(qbeg + q0 + r) * p.ldo + static_cast<size_t>(h) * kD;
      for (int c = 0; c < kD; c += 8) *reinterpret_cast<uint4*>(orow + c) = make_uint4(0, 0, 0, 0);
      if (p.lse != nullptr) p.lse[static_cast<size_t>(h) * p.Tq + qbeg + q0 + r] = -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) trace_at(p, 9, 1);
  if (warp == kProducers) tmem_dealloc(tmem, 512);
}

int attn_fwd_tc_smem_bytes() { return (1 + 2 * kStages) * kTileBytes + 1024 + 256; }

void attn_fwd_tc(const AttnParams& p, int n_tiles, int* status, cudaStream_t st) {
  if (n_tiles == 0) return;
  static SmemOptIn opt;
  opt.ensure(attn_fwd_tc_kernel, attn_fwd_tc_smem_bytes());
  attn_fwd_tc_kernel<<<dim3(n_tiles, p.Hq), kThreads, attn_fwd_tc_smem_bytes(), st>>>(p, status);
}

}  // namespace octo
