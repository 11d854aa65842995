// Gathered-key attention forward on tcgen05/TMEM with two query tiles per CTA.
//
// Same contract as attn_fwd in attention.cu (tree nodes / paged prefill: the query rows
// of a sequence attend to a gathered key list, bottom-right causal, GQA), head_dim 128.
//
// CTA = 256 query rows (tiles A = rows q0..q0+127 and B = q0+128..q0+255) of one
// sequence and one head, 384 threads in three warpgroups:
//   warp 0      TMA loads of the two Q tiles (rows are contiguous)
//   warp 1      TMEM owner and single-thread MMA issuer (event loop, below)
//   warps 2-3   K/V producers, 64 key rows each: when the warp's 64 rows are consecutive
//               in the key list (the common case: tree paths are runs of node rows) one
//               lane issues two TMA tile loads per operand; otherwise the warp gathers the
//               rows with cp.async.  Either way the stage's mbarrier counts 64 arrivals.
//   warps 4-7   softmax of tile A, warps 8-11 softmax of tile B (thread = query row)
// K and V have separate 2-stage rings and barriers: a K stage is refilled as soon as both
// S = Q K^T products of its key tile have completed, before the P V products need V.
//
// TMEM (512 columns): S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512).  P (bf16)
// is written over the first 64 columns of its S; so S_x(j+1) is issued only after
// P_x(j) V_j has completed.  The two tiles ping-pong on the tensor core: while the softmax
// warps of one tile exponentiate, the MMAs of the other run.  Issue order per tile x:
//   S_x(j) needs K_j landed and P_x(j-1) V_{j-1} complete
//   P_x(j) V_j needs S_x(j) issued, V_j landed and the softmax's P_x(j) written
// Softmax: online, exp2 domain on the SFU (ex2.approx), lazy rescale (O_x rescaled in TMEM only when the running
// max grows by more than 2^8; the rescale runs before P_x(j) is published, when
// P_x(j-1) V_{j-1} is known complete).  Epilogue O / l -> bf16 rows + natural-log lse.
//
// All waits are bounded (common.cuh): on a timeout the CTA records an error, drains its
// MMAs and copies, frees TMEM and exits.
//
// Reference parity (behaviour): the tree / packed-causal attention the reference trains
// through `octopus/rl/prefix_tree.py` (ancestor-path keys, own rows last, causal within a
// node) with FlashAttention-style online softmax.
#include <cuda.h>
#include <cuda_bf16.h>

#include "attention.h"
#include "common.cuh"

namespace octo {

namespace {

constexpr int kBM = 128, kBN = 128, kD = 128;
constexpr int kHalf = 128 * 128;       // bytes of one 64-column SW128 half of a 128-row tile
constexpr int kTile = 2 * kHalf;       // 32 KB: a 128 x 128 bf16 tile
constexpr int kStages = 2;
constexpr int kThreads = 384;
constexpr int kProdRows = 64;          // key rows per producer warp
constexpr uint32_t kColS0 = 0, kColO0 = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ uint32_t toff(int r, int c) {
  // row r, 16-byte chunk c (0..15) of a 128 x 128 bf16 tile made of two SW128 halves
  return static_cast<uint32_t>((c >> 3) * kHalf + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

struct Tiles2 {
  int rows[2];  // valid query rows of tile A / B (0: absent)
  int nend[2];  // keys visible to the tile's last row
  int nt[2];    // key tiles of the tile
};

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_pp_kernel(const __grid_constant__ AttnMaps maps, AttnParams p, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = smem;                       // 2 tiles
  uint8_t* sK = sQ + 2 * kTile;             // kStages tiles
  uint8_t* sV = sK + kStages * kTile;       // kStages tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kStages * kTile);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;            // [kStages]
  uint64_t* v_full = k_full + kStages;      // [kStages]
  uint64_t* k_empty = v_full + kStages;     // [kStages]
  uint64_t* v_empty = k_empty + kStages;    // [kStages]
  uint64_t* s_full = v_empty + kStages;     // [2] per query tile
  uint64_t* p_full = s_full + 2;            // [2]
  uint64_t* pv_done = p_full + 2;           // [2]
  uint64_t* drain = pv_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid.x = tile * Hq + head: consecutive CTAs share a key list (and, within a GQA group,
  // the K/V rows) in L2
  const int tile = blockIdx.x / p.Hq;
  const int h = blockIdx.x - tile * p.Hq;
  const int seq = p.tiles[2 * tile];
  const int q0 = p.tiles[2 * tile + 1];
  const int kvh = h / (p.Hq / p.Hkv);
  const int qbeg = p.cu_q[seq], nq = p.cu_q[seq + 1] - qbeg;
  const int kbeg = p.cu_k[seq], nk = p.cu_k[seq + 1] - kbeg;
  const int off = nk - nq;
  Tiles2 T;
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const int r = min(kBM, nq - (q0 + x * kBM));
    T.rows[x] = r > 0 ? r : 0;
    int e = T.rows[x] == 0 ? 0 : (p.causal ? min(nk, q0 + x * kBM + T.rows[x] + off) : nk);
    T.nend[x] = e > 0 ? e : 0;
    T.nt[x] = (T.nend[x] + kBN - 1) / kBN;
  }
  const int nt = max(T.nt[0], T.nt[1]);
  const int n_end_all = max(T.nend[0], T.nend[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 2 * 32);
      mbar_init(&v_full[s], 2 * 32);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 4);
      mbar_init(&pv_done[x], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&maps.q);
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
    // ------------------------------------------------------------ Q (TMA)
    if (lane == 0 && nt > 0) {
      const uint32_t bytes = (T.rows[1] > 0 ? 2u : 1u) * kTile;
      mbar_arrive_expect_tx(q_full, bytes);
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (T.rows[x] == 0) continue;
#pragma unroll
        for (int half = 0; half < 2; ++half)
          tma_load_2d(sQ + x * kTile + half * kHalf, &maps.q, q_full, h * kD + half * 64, qbeg + q0 + x * kBM);
      }
      // (a timed-out CTA still lets these land before TMEM / SMEM are released)
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(q_full, 0)) {
        if (globaltimer_ns() - t0 > OCTO_WAIT_NS) break;
      }
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ K / V producers
    const int rbase = (warp - 2) * kProdRows;   // this warp's rows of every key tile
    const __nv_bfloat16* kb = p.k + static_cast<size_t>(kvh) * kD;
    const __nv_bfloat16* vb = p.v + static_cast<size_t>(kvh) * kD;
    const int32_t* kidx = p.key_idx + kbeg;
    const int first = nk > 0 ? kidx[0] : 0;
    const int cl = lane & 15;  // 16 lanes per row: coalesced 256-byte row reads
    int nx[2];
    auto load_idx = [&](int j, int (&dst)[2]) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int kk = j * kBN + rbase + q * 32 + lane;
        dst[q] = kk < n_end_all ? static_cast<int>(kidx[kk]) : first;
      }
    };
    // one operand's 64 rows of stage `dst`: two TMA boxes when consecutive, else cp.async
    auto load_rows = [&](uint8_t* dst, const CUtensorMap* map, const __nv_bfloat16* src, uint64_t* bar,
                         bool contig, int base, const int (&ix)[2]) {
      if (contig) {
        if (lane == 0) {
          mbar_arrive_expect_tx(bar, 2u * kProdRows * 128u);
#pragma unroll
          for (int half = 0; half < 2; ++half)
            tma_load_2d(dst + half * kHalf + rbase * 128, map, bar, kvh * kD + half * 64, base);
        } else {
          mbar_arrive(bar);
        }
      } else {
        const uint32_t sbase = smem_u32(dst);
#pragma unroll
        for (int i = 0; i < kProdRows / 2; ++i) {
          const int rl = 2 * i + (lane >> 4);
          const int64_t row = static_cast<int64_t>(__shfl_sync(0xffffffffu, ix[rl >> 5], rl & 31));
          cp_async16(sbase + toff(rbase + rl, cl), src + row * p.ldk + cl * 8);
        }
        cp_async_arrive(bar);
      }
    };
    int issued_k = -1, issued_v = -1;  // last tile index loaded into each ring
    bool ok = true;
    if (nt > 0) load_idx(0, nx);
    for (int j = 0; j < nt && ok; ++j) {
      const int st = j % kStages;
      const uint32_t ph = static_cast<uint32_t>((j / kStages) & 1);
      int ix[2] = {nx[0], nx[1]};
      if (j + 1 < nt) load_idx(j + 1, nx);
      const int base = __shfl_sync(0xffffffffu, ix[0], 0);
      bool c = true;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int kk = j * kBN + rbase + q * 32 + lane;
        if (kk < n_end_all && ix[q] != base + q * 32 + lane) c = false;
      }
      const bool contig = __all_sync(0xffffffffu, c);
      if (lane == 0) ok = mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, status, 800 + st);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      load_rows(sK + st * kTile, &maps.k, kb, &k_full[st], contig, base, ix);
      issued_k = j;
      if (lane == 0) ok = mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, status, 810 + st);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      load_rows(sV + st * kTile, &maps.v, vb, &v_full[st], contig, base, ix);
      issued_v = j;
    }
    if (!ok) {
      // drain: the copies this warp issued must land before the CTA releases its memory
      asm volatile("cp.async.wait_all;" ::: "memory");
      if (lane == 0) {
        const uint64_t t0 = globaltimer_ns();
        for (int j = max(0, issued_k - 1); j <= issued_k; ++j)
          while (!mbar_try_wait(&k_full[j % kStages], (j / kStages) & 1))
            if (globaltimer_ns() - t0 > OCTO_WAIT_NS) break;
        for (int j = max(0, issued_v - 1); j <= issued_v; ++j)
          while (!mbar_try_wait(&v_full[j % kStages], (j / kStages) & 1))
            if (globaltimer_ns() - t0 > OCTO_WAIT_NS) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (event loop)
    if (lane == 0 && nt > 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(kBM, kBN, false, false, true);
      constexpr uint32_t idesc_o = umma_idesc_f16(kBM, kD, false, true, true);
      bool ok = mbar_wait(q_full, 0, abort_flag, status, 820);
      int ns[2] = {0, 0}, np[2] = {0, 0};  // next S / P.V tile per query tile
      int k_rel = 0, v_rel = 0;            // next K / V stage release
      bool issued = false;
      uint64_t t_last = globaltimer_ns();
      while (ok && (np[0] < T.nt[0] || np[1] < T.nt[1])) {
        bool progressed = false;
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          // P_x(j) V_j
          const int jp = np[x];
          if (jp < T.nt[x] && jp < ns[x] && mbar_test(&v_full[jp % kStages], (jp / kStages) & 1) &&
              mbar_test(&p_full[x], jp & 1)) {
            tc_fence_after();
            fence_proxy_async_smem();  // cp.async-gathered rows -> tensor-core reads
            const uint32_t vaddr = smem_u32(sV + (jp % kStages) * kTile);
#pragma unroll
            for (int kk = 0; kk < kBN / 16; ++kk) {
              const uint64_t bd = umma_smem_desc(vaddr + kk * 2048, kHalf, 1024);
              umma_f16_ts(tmem + kColO0 + x * 128, tmem + kColS0 + x * 128 + kk * 8, bd, idesc_o,
                          (jp > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(&pv_done[x]);
            np[x] = jp + 1;
            issued = progressed = true;
          }
          // S_x(j) = Q_x K_j^T
          const int js = ns[x];
          if (js < T.nt[x] && js == np[x] && mbar_test(&k_full[js % kStages], (js / kStages) & 1) &&
              (js == 0 || mbar_test(&pv_done[x], (js - 1) & 1))) {
            tc_fence_after();
            fence_proxy_async_smem();
            const uint32_t qaddr = smem_u32(sQ + x * kTile);
            const uint32_t kaddr = smem_u32(sK + (js % kStages) * kTile);
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t o16 = (kk >> 2) * kHalf + (kk & 3) * 32;
              umma_f16_ss(tmem + kColS0 + x * 128, umma_smem_desc(qaddr + o16, 16, 1024),
                          umma_smem_desc(kaddr + o16, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[x]);
            ns[x] = js + 1;
            issued = progressed = true;
          }
        }
        // release K / V stages whose products have all been issued (the commit fires when
        // those MMAs complete)
        while (k_rel < nt && (k_rel >= T.nt[0] || ns[0] > k_rel) && (k_rel >= T.nt[1] || ns[1] > k_rel)) {
          umma_commit(&k_empty[k_rel % kStages]);
          ++k_rel;
        }
        while (v_rel < nt && (v_rel >= T.nt[0] || np[0] > v_rel) && (v_rel >= T.nt[1] || np[1] > v_rel)) {
          umma_commit(&v_empty[v_rel % kStages]);
          ++v_rel;
        }
        if (progressed) {
          t_last = globaltimer_ns();
        } else if (*abort_flag) {
          ok = false;
        } else if (globaltimer_ns() - t_last > wait_budget_ns(status)) {
          *abort_flag = 1;
          record_error(status, kErrMbarTimeout, 830);
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
    // ------------------------------------------------------------ softmax + epilogue
    const int x = (warp - 4) >> 2;              // query tile
    const int quarter = warp & 3;               // TMEM lane quarter of this warp
    const int r = quarter * 32 + lane;          // TMEM lane = query row in the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t colS = kColS0 + x * 128, colO = kColO0 + x * 128;
    const int qi = q0 + x * kBM + r;            // sequence-relative query index
    const int ntx = T.nt[x];
    const int lim = p.causal ? min(T.nend[x], qi + off + 1) : T.nend[x];
    const float sc = p.scale * kLog2e;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntx; ++j) {
      if (!mbar_wait(&s_full[x], j & 1, abort_flag, status, 840 + x)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kBN];
      {
        uint32_t v0[32], v1[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + colS, v0);
        tmem_ld_32x32b_x32(tmem + lane_addr + colS + 32, v1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = __uint_as_float(v0[i]);
          s[32 + i] = __uint_as_float(v1[i]);
        }
        tmem_ld_32x32b_x32(tmem + lane_addr + colS + 64, v0);
        tmem_ld_32x32b_x32(tmem + lane_addr + colS + 96, v1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[64 + i] = __uint_as_float(v0[i]);
          s[96 + i] = __uint_as_float(v1[i]);
        }
      }
      const int kbase = j * kBN;
      if (kbase + kBN > lim) {
#pragma unroll
        for (int i = 0; i < kBN; ++i)
          if (kbase + i >= lim) s[i] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < kBN; ++i) mx = fmaxf(mx, s[i]);
      mx *= sc;
      float alpha = 1.f;
      if (j == 0) {
        m = mx;
      } else if (mx > m + kRescaleThreshold) {
        alpha = exp2f(m - mx);
        m = mx;
      }
      const float mref = m == -INFINITY ? 0.f : m;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float a = exp2_approx(fmaf(s[c * 32 + 2 * i], sc, -mref));
          const float b = exp2_approx(fmaf(s[c * 32 + 2 * i + 1], sc, -mref));
          rs += a + b;
          pk[i] = pack_bf16x2(a, b);
        }
        // P chunk c -> columns [16c, 16c + 16) of S: S columns < 32(c + 1) are already in registers
        tmem_st_32x32b_x16(tmem + lane_addr + colS + c * 16, pk);
      }
      l = l * alpha + rs;
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
        // P_x(j-1) V_{j-1} has completed: S_x(j) was issued after it
#pragma unroll 1
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + lane_addr + colO + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
          tmem_st_32x32b_x32(tmem + lane_addr + colO + c * 32, v);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    // epilogue: O / l
    const bool write = r < T.rows[x];
    const size_t orow_off = static_cast<size_t>(qbeg + q0 + x * kBM + (write ? r : 0)) * p.ldo +
                            static_cast<size_t>(h) * kD;
    if (ok && ntx > 0 && mbar_wait(&pv_done[x], (ntx - 1) & 1, abort_flag, status, 850 + x)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + orow_off;
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + colO + c * 32, v);
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
        p.lse[static_cast<size_t>(h) * p.Tq + qbeg + q0 + x * kBM + r] = l > 0.f ? (m + log2f(l)) * kLn2 : -INFINITY;
    } else if (ntx == 0 && write) {
      __nv_bfloat16* orow = p.o + orow_off;
      for (int c = 0; c < kD; c += 8) *reinterpret_cast<uint4*>(orow + c) = make_uint4(0, 0, 0, 0);
      if (p.lse != nullptr) p.lse[static_cast<size_t>(h) * p.Tq + qbeg + q0 + x * kBM + r] = -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

int attn_fwd_pp_smem_bytes() { return (2 + 2 * kStages) * kTile + 1024 + 256; }

void attn_fwd_pp(const AttnParams& p, const AttnMaps& maps, int n_tiles, int* status, cudaStream_t st) {
  if (n_tiles == 0) return;
  static SmemOptIn opt;
  opt.ensure(attn_fwd_pp_kernel, attn_fwd_pp_smem_bytes());
  attn_fwd_pp_kernel<<<n_tiles * p.Hq, kThreads, attn_fwd_pp_smem_bytes(), st>>>(maps, p, status);
}

}  // namespace octo
