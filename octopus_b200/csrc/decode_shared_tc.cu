// Shared-prefix ("cascade") paged decode attention on tcgen05/TMEM (sm_100a).
//
// Same plan tables and partial format as decode_shared.cu: a work item is (segment, key
// chunk, kv head); a segment is a key range shared by up to kSegRows decode rows (or one
// row's own, growing remainder).  Here the 128 TMEM lanes of one MMA tile hold the
// segment's (row, GQA head) pairs, lane = row * G + head, so up to 128 / G rows (16 for
// G = 7) share every K/V tile the item streams:
//   S = Q K_j^T     tcgen05.mma M=128 (row, head) x N=64 keys x K=128, SMEM operands
//   P = softmax     thread = TMEM lane, online in the exp2 domain with lazy rescaling
//   O += P V_j      A = P (bf16, written over S in TMEM), B = V_j (SMEM, MN-major)
// and each (row, head) lane writes its normalised partial (o, lse) to the row's slot for
// the item; decode_shared_combine_kernel merges a row's slots.
//
// CTA (192 threads, two per SM): warp 0 producer (item descriptor -> SMEM ring, 64-key K/V
// tiles by two TMA boxes per operand when the slots are consecutive, else cp.async), warp 1
// TMEM owner + single-thread MMA issuer (event loop; S double-buffered so S_{j+1} overlaps
// the softmax of j), warps 2-5 softmax and epilogue; each softmax thread also writes its
// lane's Q row (16 independent 16-byte loads) at the start of an item.  The descriptor (a
// chain of dependent table loads) is resolved once, by the producer, while the previous
// item streams.
// TMEM (256 columns per CTA): S[0] [0,64), S[1] [64,128), O [128,256).
// All waits are bounded (common.cuh); a timed-out CTA records an error, drains and frees TMEM.
#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "decode_shared.h"

namespace octo {

namespace {

constexpr int kTileK = 64;                // keys per tile
constexpr int kHalf64 = 64 * 128;         // 8 KB: 64-column SW128 half of a 64-row tile
constexpr int kKVBytes = 4 * kHalf64;     // K (2 halves) + V (2 halves)
constexpr int kQHalf = 128 * 128;         // 16 KB: 64-column half of the 128-lane Q tile
constexpr int kQBytes = 2 * kQHalf;
constexpr int kThreads = 192;
constexpr uint32_t kColS = 0, kColO = 128, kTmemCols = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;

struct ItemDesc {
  int ntiles, nkeys, kvh, nrows;
  int start, k0, pad0, pad1;
  int rows[kSegRows];
  int slot[kSegRows];
};

__device__ __forceinline__ uint32_t off64(int r, int c) {  // 64-row tile, 16-byte chunk c
  return static_cast<uint32_t>((c >> 3) * kHalf64 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint32_t offq(int r, int c) {   // 128-lane Q tile
  return static_cast<uint32_t>((c >> 3) * kQHalf + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// event trace of CTA 0 (p.trace != nullptr): [event * 64 + tile] = globaltimer
__device__ __forceinline__ void trace_at(const DecodeSharedParams& p, int ev, int t) {
  if (p.trace != nullptr && blockIdx.x == 0 && t < 64) p.trace[ev * 64 + t] = globaltimer_ns();  // ev < 10
}

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > OCTO_WAIT_NS) break;
}

}  // namespace

// kStages K/V stages; kMinBlocks CTAs per SM
template <int kStages, int kMinBlocks>
__global__ void __launch_bounds__(kThreads, kMinBlocks)
    decode_shared_tc_kernel(const __grid_constant__ DecodeSharedMaps maps, DecodeSharedParams p, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + kQBytes;  // [kStages]
  ItemDesc* desc = reinterpret_cast<ItemDesc*>(sKV + kStages * kKVBytes);  // [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(desc + 2);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;       // [kStages]
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* s_full = kv_empty + kStages;  // [2]
  uint64_t* p_full = s_full + 2;          // [2]
  uint64_t* pv_done = p_full + 2;         // [2]
  uint64_t* desc_full = pv_done + 2;      // [2]
  uint64_t* desc_empty = desc_full + 2;   // [2]
  uint64_t* drain = desc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.n_items[0];
  const int ck = p.n_items[1];
  const int G = p.Hq / p.Hkv;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 4);  // the 4 softmax warps, after writing their lanes' Q rows
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 32);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 4);
      mbar_init(&pv_done[b], 1);
      mbar_init(&desc_full[b], 1);
      mbar_init(&desc_empty[b], 5);  // the MMA thread + 4 softmax warps
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&maps.k);
    tma_prefetch_desc(&maps.v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const size_t ld = static_cast<size_t>(p.Hkv) * 128;
    const int c16 = lane & 15;
    bool ok = true;
    int t = 0;           // tiles issued by this CTA (all items)
    int last_t = -1;
    for (int it = blockIdx.x, i = 0; it < n_items && ok; it += gridDim.x, ++i) {
      // descriptor of item `it` (every lane resolves the same chain; loads are broadcasts)
      const int e = p.items[it / p.Hkv];
      const int kvh = it % p.Hkv;
      const int seg = e >> 8, chunk = e & 255;
      int len = p.seg_len[seg];
      if (len < 0) len = max(0, p.kv_len[p.seg_rows[seg * kSegRows]] - p.seg_off[seg]);
      const int k0 = min(len, chunk * ck);  // ck: the plan's keys per item (device scalar)
      const int k1 = min(len, k0 + ck);
      const int start = p.seg_start[seg];
      const int myrow = lane < kSegRows ? p.seg_rows[seg * kSegRows + lane] : -1;
      const int myslot = lane < kSegRows ? p.seg_slot[seg * kSegRows + lane] + chunk : 0;
      const int nrows = __popc(__ballot_sync(0xffffffffu, myrow >= 0));
      const int ntiles = (k1 - k0 + kTileK - 1) / kTileK;
      ItemDesc* d = desc + (i & 1);
      if (lane == 0) trace_at(p, 6, i);
      if (lane == 0) ok = mbar_wait(&desc_empty[i & 1], ((i >> 1) & 1) ^ 1u, abort_flag, status, 1000);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      if (lane < kSegRows) {
        d->rows[lane] = myrow;
        d->slot[lane] = myslot;
      }
      if (lane == 0) {
        d->ntiles = ntiles;
        d->nkeys = k1 - k0;
        d->kvh = kvh;
        d->nrows = nrows;
        d->start = start;
        d->k0 = k0;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&desc_full[i & 1]);
      // K / V tiles
      const int32_t* idx = p.kv_indices + start;
      const int first = k0 < k1 ? static_cast<int>(idx[k0]) : 0;
      for (int j = 0; j < ntiles && ok; ++j, ++t) {
        const int st = t % kStages;
        const int kb = k0 + j * kTileK;
        int ix[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) ix[q] = kb + q * 32 + lane < k1 ? static_cast<int>(idx[kb + q * 32 + lane]) : first;
        const int base = __shfl_sync(0xffffffffu, ix[0], 0);
        bool c = true;
#pragma unroll
        for (int q = 0; q < 2; ++q)
          if (kb + q * 32 + lane < k1 && ix[q] != base + q * 32 + lane) c = false;
        const bool contig = __all_sync(0xffffffffu, c);
        if (lane == 0) trace_at(p, 0, t);
        if (lane == 0) ok = mbar_wait(&kv_empty[st], ((t / kStages) & 1) ^ 1u, abort_flag, status, 1002 + st);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        uint8_t* dst = sKV + st * kKVBytes;
        if (contig) {
          if (lane == 0) {
            mbar_arrive_expect_tx(&kv_full[st], static_cast<uint32_t>(kKVBytes));
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              tma_load_2d(dst + half * kHalf64, &maps.k, &kv_full[st], kvh * 128 + half * 64, base);
              tma_load_2d(dst + 2 * kHalf64 + half * kHalf64, &maps.v, &kv_full[st], kvh * 128 + half * 64, base);
            }
          } else {
            mbar_arrive(&kv_full[st]);
          }
        } else {
          const uint32_t sb = smem_u32(dst);
#pragma unroll
          for (int r2 = 0; r2 < kTileK / 2; ++r2) {
            const int r = 2 * r2 + (lane >> 4);
            const int64_t row = static_cast<int64_t>(__shfl_sync(0xffffffffu, ix[r >> 5], r & 31));
            cp_async16(sb + off64(r, c16), p.k_cache + row * ld + kvh * 128 + c16 * 8);
            cp_async16(sb + 2 * kHalf64 + off64(r, c16), p.v_cache + row * ld + kvh * 128 + c16 * 8);
          }
          cp_async_arrive(&kv_full[st]);
        }
        last_t = t;
        if (lane == 0) trace_at(p, 1, t);
      }
    }
    if (!ok) {
      asm volatile("cp.async.wait_all;" ::: "memory");
      if (lane == 0)
        for (int u = max(0, last_t - kStages + 1); u <= last_t; ++u) drain_wait(&kv_full[u % kStages], (u / kStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(128, kTileK, false, false, true);
      constexpr uint32_t idesc_o = umma_idesc_f16(128, 128, false, true, true);
      const uint32_t qaddr = smem_u32(sQ);
      bool ok = true, issued = false;
      int tb = 0;  // first CTA tile of the current item
      for (int it = blockIdx.x, i = 0; it < n_items && ok; it += gridDim.x, ++i) {
        if (!mbar_wait(&desc_full[i & 1], (i >> 1) & 1, abort_flag, status, 1010)) {
          ok = false;
          break;
        }
        const int ntiles = desc[i & 1].ntiles;
        mbar_arrive(&desc_empty[i & 1]);
        // (Q is written for every item, ntiles == 0 included, so the phases stay in step)
        if (!mbar_wait(q_full, i & 1, abort_flag, status, 1012)) {
          ok = false;
          break;
        }
        trace_at(p, 7, i);
        int js = 0, jp = 0;
        uint64_t t_last = globaltimer_ns();
        while (ok && jp < ntiles) {
          bool progressed = false;
          const int ts = tb + js, tp = tb + jp;
          // S(ts) into S[ts & 1]: K landed, and P(ts - 2) V consumed from that buffer
          if (js < ntiles && mbar_test(&kv_full[ts % kStages], (ts / kStages) & 1) &&
              (ts < 2 || mbar_test(&pv_done[ts & 1], ((ts - 2) >> 1) & 1))) {
            tc_fence_after();
            fence_proxy_async_smem();  // cp.async-written Q / K / V -> tensor-core reads
            const uint32_t kaddr = smem_u32(sKV + (ts % kStages) * kKVBytes);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t oq = (kk >> 2) * kQHalf + (kk & 3) * 32, ok_ = (kk >> 2) * kHalf64 + (kk & 3) * 32;
              umma_f16_ss(tmem + kColS + (ts & 1) * 64, umma_smem_desc(qaddr + oq, 16, 1024),
                          umma_smem_desc(kaddr + ok_, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[ts & 1]);
            trace_at(p, 2, ts);
            ++js;
            issued = progressed = true;
          }
          // O += P(tp) V(tp)
          if (jp < js && mbar_test(&p_full[tp & 1], (tp >> 1) & 1)) {
            tc_fence_after();
            const uint32_t vaddr = smem_u32(sKV + (tp % kStages) * kKVBytes + 2 * kHalf64);
#pragma unroll
            for (int kk = 0; kk < kTileK / 16; ++kk)
              umma_f16_ts(tmem + kColO, tmem + kColS + (tp & 1) * 64 + kk * 8,
                          umma_smem_desc(vaddr + kk * 2048, kHalf64, 1024), idesc_o, (jp > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&pv_done[tp & 1]);
            umma_commit(&kv_empty[tp % kStages]);
            trace_at(p, 3, tp);
            ++jp;
            issued = progressed = true;
          }
          if (progressed) {
            t_last = globaltimer_ns();
          } else if (*abort_flag) {
            ok = false;
          } else if (globaltimer_ns() - t_last > wait_budget_ns(status)) {
            *abort_flag = 1;
            record_error(status, kErrMbarTimeout, 1013);
            ok = false;
          }
        }
        tb += ntiles;
      }
      if (issued) {
        umma_commit(drain);
        drain_wait(drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3;
    const int L = quarter * 32 + lane;  // TMEM lane = row * G + head
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const float sc = p.scale * kLog2e;
    int t = 0;
    bool ok = true;
    for (int it = blockIdx.x, i = 0; it < n_items && ok; it += gridDim.x, ++i) {
      if (!mbar_wait(&desc_full[i & 1], (i >> 1) & 1, abort_flag, status, 1020)) {
        ok = false;
        break;
      }
      const ItemDesc* d = desc + (i & 1);
      const int ntiles = d->ntiles, nkeys = d->nkeys, kvh = d->kvh;
      const int jrow = L / G;
      const bool valid = jrow < d->nrows;
      const int row = valid ? d->rows[jrow] : 0;
      const int slot = valid ? d->slot[jrow] : 0;
      // this lane's Q row (row, head kvh * G + L % G): the previous item's S MMAs have all
      // completed (this warp saw their commit), so sQ is free
      if (valid) {
        const uint4* src = reinterpret_cast<const uint4*>(p.q + static_cast<size_t>(row) * p.ldq +
                                                          static_cast<size_t>(kvh * G + L % G) * 128);
        uint4 v[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) v[c] = src[c];
#pragma unroll
        for (int c = 0; c < 16; ++c) *reinterpret_cast<uint4*>(sQ + offq(L, c)) = v[c];
      }
      fence_proxy_async_smem();  // generic-proxy stores -> tensor-core reads
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&desc_empty[i & 1]);
        mbar_arrive(q_full);
      }
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < ntiles; ++j, ++t) {
        const int b = t & 1;
        if (!mbar_wait(&s_full[b], (t >> 1) & 1, abort_flag, status, 1021)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t s0[32], s1[32];
        tmem_ld_32x32b_x32(tmem + lane_addr + kColS + b * 64, s0);
        tmem_ld_32x32b_x32(tmem + lane_addr + kColS + b * 64 + 32, s1);
        tmem_wait_ld();
        if (threadIdx.x == 64) trace_at(p, 4, t);
        const int lim = nkeys - j * kTileK;  // keys of this tile that exist
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (c < lim) mx = fmaxf(mx, __uint_as_float(s0[c]));
          if (c + 32 < lim) mx = fmaxf(mx, __uint_as_float(s1[c]));
        }
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
        uint32_t pk[16];
#pragma unroll
        for (int i2 = 0; i2 < 16; ++i2) {
          const int c = 2 * i2;
          const float a = c < lim ? exp2_approx(fmaf(__uint_as_float(s0[c]), sc, -mref)) : 0.f;
          const float bb = c + 1 < lim ? exp2_approx(fmaf(__uint_as_float(s0[c + 1]), sc, -mref)) : 0.f;
          rs += a + bb;
          pk[i2] = pack_bf16x2(a, bb);
        }
        tmem_st_32x32b_x16(tmem + lane_addr + kColS + b * 64, pk);
#pragma unroll
        for (int i2 = 0; i2 < 16; ++i2) {
          const int c = 32 + 2 * i2;
          const float a = c < lim ? exp2_approx(fmaf(__uint_as_float(s1[2 * i2]), sc, -mref)) : 0.f;
          const float bb = c + 1 < lim ? exp2_approx(fmaf(__uint_as_float(s1[2 * i2 + 1]), sc, -mref)) : 0.f;
          rs += a + bb;
          pk[i2] = pack_bf16x2(a, bb);
        }
        tmem_st_32x32b_x16(tmem + lane_addr + kColS + b * 64 + 16, pk);
        if (threadIdx.x == 64) trace_at(p, 8, t);
        l = l * alpha + rs;
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          // O holds P V of the item's tiles < j: wait for the last of them, then rescale
          if (!mbar_wait(&pv_done[(t - 1) & 1], ((t - 1) >> 1) & 1, abort_flag, status, 1022)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + lane_addr + kColO + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
            tmem_st_32x32b_x32(tmem + lane_addr + kColO + c * 32, v);
          }
        }
        tmem_wait_st();
        if (threadIdx.x == 64) trace_at(p, 9, t);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[b]);
        if (threadIdx.x == 64) trace_at(p, 5, t);
      }
      if (!ok) break;
      // epilogue: normalised partial of every valid (row, head) lane
      const int hq = kvh * G + L % G;
      const size_t pbase = (static_cast<size_t>(row) * p.Hq + hq) * p.max_slots + slot;
      if (ntiles > 0) {
        if (!mbar_wait(&pv_done[(t - 1) & 1], ((t - 1) >> 1) & 1, abort_flag, status, 1023)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float* po = p.part_o + pbase * 128;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + lane_addr + kColO + c * 32, v);
          tmem_wait_ld();
          if (valid) {
#pragma unroll
            for (int g4 = 0; g4 < 8; ++g4)
              *reinterpret_cast<float4*>(po + c * 32 + g4 * 4) =
                  make_float4(__uint_as_float(v[g4 * 4]) * inv, __uint_as_float(v[g4 * 4 + 1]) * inv,
                              __uint_as_float(v[g4 * 4 + 2]) * inv, __uint_as_float(v[g4 * 4 + 3]) * inv);
          }
        }
        // (O is read: the next item's first P V may overwrite it once this warp's next P lands)
        tc_fence_before();
        if (valid) p.part_lse[pbase] = l > 0.f ? m + log2f(l) : -INFINITY;
      } else if (valid) {
        float* po = p.part_o + pbase * 128;
        for (int c = 0; c < 128; c += 4) *reinterpret_cast<float4*>(po + c) = make_float4(0.f, 0.f, 0.f, 0.f);
        p.part_lse[pbase] = -INFINITY;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <int kStages>
static int smem_bytes() {
  return kQBytes + kStages * kKVBytes + 2 * static_cast<int>(sizeof(ItemDesc)) + 256 + 1024;
}
int decode_shared_tc_smem_bytes() { return smem_bytes<2>(); }

template <int kStages, int kMinBlocks>
static void launch(const DecodeSharedParams& p, const DecodeSharedMaps& maps, int sms, int* status,
                   cudaStream_t st) {
  auto kern = decode_shared_tc_kernel<kStages, kMinBlocks>;
  static SmemOptIn opt;
  opt.ensure(kern, smem_bytes<kStages>());
  kern<<<kMinBlocks * sms, kThreads, smem_bytes<kStages>(), st>>>(maps, p, status);
}

void decode_shared_tc_launch(const DecodeSharedParams& p, const DecodeSharedMaps& maps, int sms, int* status,
                             cudaStream_t st) {
  // two CTAs per SM with two K/V stages each: measured faster than one CTA with four stages
  // (two item streams hide each other's boundaries)
  launch<2, 2>(p, maps, sms, status, st);
  decode_shared_combine(p, st);
}

}  // namespace octo
