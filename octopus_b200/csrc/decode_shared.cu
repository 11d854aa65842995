// Shared-prefix ("cascade") paged decode attention (sm_100a).
//
// Decode rows of a multi-agent rollout share long key prefixes: every agent of a task
// mounts the task prefix, forked threads share their parent's context.  Attending row by
// row streams those shared keys once per row.  Here the host splits every row's key
// list into segments: a segment is a key range [start, start + len) of the index list
// shared by up to kSegRows rows (the rows' contexts agree on it), or a row's own
// remainder (dynamic length: grows by one key per decode step, read from kv_len).
// A work item is (segment, key chunk, kv head).  (decode_shared_tc.cu is the tcgen05
// variant of this kernel with up to 128 / G rows per segment.)  Its K/V tiles are gathered once into
// SMEM by the producer warp and used by every row of the segment: two consumer warps,
// each holding the GQA query heads of 16 / G rows in the 16 rows of an mma.sync tile
// (for G = 7, two rows per warp fill 14 of 16 tile rows instead of 7).  Each item
// writes a partial (o, lse) per (row, head) into the row's slot for that (segment,
// chunk); a combine kernel merges a row's slots.
//
// All tables (segments, items, slot counts) are device arrays and the item count is a
// device scalar, so one launch configuration serves every decode step of a CUDA graph
// while the host re-plans between generate calls.
//
// mbarrier waits are bounded (common.cuh); a timeout records an error and stops the CTA.
#include <cuda_bf16.h>

#include "common.cuh"
#include "decode_shared.h"

namespace octo {

namespace {

constexpr int kTile = 64;                       // keys per SMEM tile
constexpr int kStages = 3;
constexpr int kHalfBytes = kTile * 128;
constexpr int kTileBytes = 4 * kHalfBytes;      // K (2 swizzle halves) + V (2 halves)
constexpr int kConsumers = 2;
constexpr float kLog2e = 1.4426950408889634f;

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
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
  return static_cast<uint32_t>((c >> 3) * kHalfBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

struct SItem {
  int seg, kvh, k0, k1;  // keys [k0, k1) of the segment (segment-relative)
  int start;             // index-list offset of segment key 0
  int chunk;
};

__device__ __forceinline__ SItem sitem_of(const DecodeSharedParams& p, int it) {
  SItem x;
  const int e = p.items[it / p.Hkv];
  x.kvh = it % p.Hkv;
  x.seg = e >> 8;
  x.chunk = e & 255;
  int len = p.seg_len[x.seg];
  if (len < 0) len = max(0, p.kv_len[p.seg_rows[x.seg * kSegRows]] - p.seg_off[x.seg]);
  const int ck = p.n_items[1];  // (device scalar: graph-safe across plans)
  x.k0 = min(len, x.chunk * ck);
  x.k1 = min(len, x.k0 + ck);
  x.start = p.seg_start[x.seg];
  return x;
}

}  // namespace

__global__ void __launch_bounds__(32 * (1 + kConsumers), 2) decode_shared_kernel(DecodeSharedParams p, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kTileBytes);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.n_items[0];

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 32);
      mbar_init(&empty[s], kConsumers);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------ producer warp
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    const size_t ld = static_cast<size_t>(p.Hkv) * 128;
    const int c = lane & 15;
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
      const SItem x = sitem_of(p, it);
      const int32_t* idx = p.kv_indices + x.start;
      const int first = x.k0 < x.k1 ? static_cast<int>(idx[x.k0]) : 0;
      // slot indices of the next tile are loaded one tile ahead (their latency hides
      // behind the current tile's wait and copies)
      int n0 = x.k0 + lane < x.k1 ? static_cast<int>(idx[x.k0 + lane]) : first;
      int n1 = x.k0 + 32 + lane < x.k1 ? static_cast<int>(idx[x.k0 + 32 + lane]) : first;
      for (int t0 = x.k0; t0 < x.k1; t0 += kTile) {
        int i0 = n0, i1 = n1;
        if (p.n_slots > 0) {
          if (!index_ok(i0, p.n_slots, status, 730)) i0 = 0;
          if (!index_ok(i1, p.n_slots, status, 731)) i1 = 0;
        }
        if (t0 + kTile < x.k1) {
          const int u = t0 + kTile;
          n0 = u + lane < x.k1 ? static_cast<int>(idx[u + lane]) : first;
          n1 = u + 32 + lane < x.k1 ? static_cast<int>(idx[u + 32 + lane]) : first;
        }
        if (lane == 0 && !mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status, 720 + stage)) ok = false;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        const uint32_t base = smem_u32(smem + stage * kTileBytes);
#pragma unroll
        for (int i = 0; i < kTile / 2; ++i) {
          const int r = 2 * i + (lane >> 4);
          const int64_t row = static_cast<int64_t>(__shfl_sync(0xffffffffu, i < 16 ? i0 : i1, r & 31));
          cp_async16(base + tile_off(r, c), p.k_cache + row * ld + x.kvh * 128 + c * 8);
          cp_async16(base + 2 * kHalfBytes + tile_off(r, c), p.v_cache + row * ld + x.kvh * 128 + c * 8);
        }
        cp_async_arrive(&full[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ consumer warps
    const int w = warp - 1;
    const int G = p.Hq / p.Hkv;
    const int R = 16 / G;                 // rows per consumer tile
    const int g = lane >> 2, t4 = lane & 3;
    const float sc = p.scale * kLog2e;
    int stage = 0;
    uint32_t phase = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      const SItem x = sitem_of(p, it);
      // tile rows t -> (segment row w * R + t / G, head t % G); rows past the segment are zero
      int rb[2], hh[2], sr[2];
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int t = g + 8 * hr;
        const int j = t / G;
        sr[hr] = w * R + j;
        hh[hr] = t - j * G;
        rb[hr] = (j < R && sr[hr] < kSegRows) ? p.seg_rows[x.seg * kSegRows + sr[hr]] : -1;
      }
      const bool any = __any_sync(0xffffffffu, rb[0] >= 0 || rb[1] >= 0);
      uint32_t qf[8][4];
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int cc = kk * 16 + t4 * 2;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          if (rb[hr] >= 0) {
            const __nv_bfloat16* qr =
                p.q + static_cast<size_t>(rb[hr]) * p.ldq + static_cast<size_t>(x.kvh * G + hh[hr]) * 128;
            qf[kk][hr] = *reinterpret_cast<const uint32_t*>(qr + cc);
            qf[kk][hr + 2] = *reinterpret_cast<const uint32_t*>(qr + cc + 8);
          } else {
            qf[kk][hr] = 0u;
            qf[kk][hr + 2] = 0u;
          }
        }
      }
      float o[16][4];
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
      bool ok = true;
      for (int t0 = x.k0; t0 < x.k1; t0 += kTile) {
        if (!mbar_wait(&full[stage], phase, abort_flag, status, 820 + stage)) {
          ok = false;
          break;
        }
        if (any) {
          const uint32_t sK = smem_u32(smem + stage * kTileBytes);
          const uint32_t sV = sK + 2 * kHalfBytes;
          float s[8][4];
#pragma unroll
          for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {
              uint32_t b0, b1, b2, b3;
              const int r = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
              const int cc = kk * 2 + ((lane >> 3) & 1);
              ldsm_x4(sK + tile_off(r, cc), b0, b1, b2, b3);
              mma_bf16(s[2 * jp], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
              mma_bf16(s[2 * jp + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
            }
          }
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            float mx = mrow[hr];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int kj = t0 + j * 8 + t4 * 2 + e;
                float v = s[j][hr * 2 + e] * sc;
                if (kj >= x.k1) v = -INFINITY;
                s[j][hr * 2 + e] = v;
                mx = fmaxf(mx, v);
              }
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mref = mx == -INFINITY ? 0.f : mx;
            const float corr = exp2f(mrow[hr] - mref);
            mrow[hr] = mx;
            float rs = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float pv = exp2_approx(s[j][hr * 2 + e] - mref);
                s[j][hr * 2 + e] = pv;
                rs += pv;
              }
            }
            lrow[hr] = lrow[hr] * corr + rs;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              o[i][hr * 2] *= corr;
              o[i][hr * 2 + 1] *= corr;
            }
          }
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t a0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
            const uint32_t a1 = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
            const uint32_t a2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            const uint32_t a3 = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int dp = 0; dp < 8; ++dp) {
              uint32_t b0, b1, b2, b3;
              const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
              const int cc = dp * 2 + (lane >> 4);
              ldsm_x4_t(sV + tile_off(r, cc), b0, b1, b2, b3);
              mma_bf16(o[2 * dp], a0, a1, a2, a3, b0, b1);
              mma_bf16(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float l = lrow[hr];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        if (rb[hr] < 0) continue;
        const int b = rb[hr];
        const int hq = x.kvh * G + hh[hr];
        const int slot = p.seg_slot[x.seg * kSegRows + sr[hr]] + x.chunk;
        const size_t base = (static_cast<size_t>(b) * p.Hq + hq) * p.max_slots + slot;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float* po = p.part_o + base * 128;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          *reinterpret_cast<float2*>(po + i * 8 + t4 * 2) = make_float2(o[i][hr * 2] * inv, o[i][hr * 2 + 1] * inv);
        if (t4 == 0) p.part_lse[base] = l > 0.f ? mrow[hr] + log2f(l) : -INFINITY;
      }
    }
  }
}

// o[b, hq] = merge over the row's slots (lse in log2 units)
__global__ void decode_shared_combine_kernel(DecodeSharedParams p) {
  grid_dep_launch();
  const int b = blockIdx.x, hq = blockIdx.y;
  const int ns = p.row_nslot[b];
  const size_t base = (static_cast<size_t>(b) * p.Hq + hq) * p.max_slots;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, p.part_lse[base + s]);
  const float mref = M == -INFINITY ? 0.f : M;
  for (int c = threadIdx.x; c < 128; c += blockDim.x) {
    float L = 0.f, acc = 0.f;
    for (int s = 0; s < ns; ++s) {
      const float w = exp2f(p.part_lse[base + s] - mref);
      L += w;
      acc += w * p.part_o[(base + s) * 128 + c];
    }
    p.o[static_cast<size_t>(b) * p.ldo + static_cast<size_t>(hq) * 128 + c] =
        __float2bfloat16(L > 0.f ? acc / L : 0.f);
  }
}

int decode_shared_smem_bytes() { return kStages * kTileBytes + 1024 + 2 * kStages * 8 + 16; }

void decode_shared_launch(const DecodeSharedParams& p, int grid, int* status, cudaStream_t st) {
  static SmemOptIn opt;
  opt.ensure(decode_shared_kernel, decode_shared_smem_bytes());
  decode_shared_kernel<<<grid, 32 * (1 + kConsumers), decode_shared_smem_bytes(), st>>>(p, status);
  decode_shared_combine(p, st);
}

void decode_shared_combine(const DecodeSharedParams& p, cudaStream_t st) {
  decode_shared_combine_kernel<<<dim3(p.B, p.Hq), 128, 0, st>>>(p);
}

}  // namespace octo
