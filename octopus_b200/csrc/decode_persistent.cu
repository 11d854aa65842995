// Persistent paged decode attention (sm_100a).
//
// One query row per request, keys/values gathered from a page-size-1 KV cache by slot
// index.  Work items are (request, kv head, key split); a persistent CTA streams the
// K/V tiles of its items through a multi-stage SMEM ring filled by a producer warp
// (cp.async row gathers into a 128-byte XOR-swizzled layout, completion tracked on an
// mbarrier with cp.async.mbarrier.arrive), so the copy pipeline never drains between
// items.  The consumer warp packs the GQA group's query heads into the
// 16 rows of an mma.sync tile, runs the online softmax in the exp2 domain, and writes a
// partial (o, lse) per item; a combine kernel merges the splits.
//
// Items are ordered (split, kv head, request) so CTAs working at the same time read
// the same key range of consecutive requests: requests that share a prefix of slots
// (a mounted task prefix, a forked parent) then hit those pages in L2.
//
// Every mbarrier wait is bounded (common.cuh): on timeout the CTA records an error in
// the status word and stops.
#include <cuda_bf16.h>

#include "common.cuh"
#include "decode_persistent.h"

namespace octo {

namespace {

constexpr int kTile = 64;        // keys per tile
constexpr int kStages = 3;       // SMEM ring depth (2 CTAs per SM)
constexpr int kHalfBytes = kTile * 128;          // 64 rows x 64 cols bf16 (one swizzle column half)
constexpr int kTileBytes = 4 * kHalfBytes;       // K (2 halves) + V (2 halves) = 32 KB


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

// Byte offset of (row r, 16-byte chunk c in 0..15) of a K or V tile made of two
// 128-byte-swizzled column halves (chunks 0-7 in half 0, 8-15 in half 1).
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
  return static_cast<uint32_t>((c >> 3) * kHalfBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

struct Item {
  int b, kvh, split, k0, k1;
};

__device__ __forceinline__ Item item_of(const DecodePersistParams& p, int it) {
  Item x;
  x.b = it % p.B;
  const int rest = it / p.B;
  x.kvh = rest % p.Hkv;
  x.split = rest / p.Hkv;
  const int nk = p.kv_len[x.b];
  const int per = ((nk + p.num_splits - 1) / p.num_splits + kTile - 1) / kTile * kTile;
  x.k0 = min(nk, x.split * per);
  x.k1 = min(nk, x.k0 + per);
  return x;
}

constexpr float kLog2e = 1.4426950408889634f;

}  // namespace

__global__ void __launch_bounds__(64, 2) decode_persistent_kernel(DecodePersistParams p, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kTileBytes);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.B * p.Hkv * p.num_splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 32);  // one completion arrival per producer lane
      mbar_init(&empty[s], 1);
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
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
      const Item x = item_of(p, it);
      const int32_t* idx = p.kv_indices + p.kv_start[x.b];
      const int first = x.k0 < x.k1 ? static_cast<int>(idx[x.k0]) : 0;
      // the tile's 64 slot indices: one coalesced load per lane (rows lane, lane + 32),
      // handed to the copying lanes by shuffle (no dependent load per row); loaded one
      // tile ahead so their latency hides behind the current tile's wait and copies
      int n0 = x.k0 + lane < x.k1 ? static_cast<int>(idx[x.k0 + lane]) : first;
      int n1 = x.k0 + 32 + lane < x.k1 ? static_cast<int>(idx[x.k0 + 32 + lane]) : first;
      for (int t0 = x.k0; t0 < x.k1; t0 += kTile) {
        const int i0 = n0, i1 = n1;
        if (t0 + kTile < x.k1) {
          const int u = t0 + kTile;
          n0 = u + lane < x.k1 ? static_cast<int>(idx[u + lane]) : first;
          n1 = u + 32 + lane < x.k1 ? static_cast<int>(idx[u + 32 + lane]) : first;
        }
        if (lane == 0) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status, 700 + stage)) ok = false;
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        // 16 lanes per cache row (one 16-byte chunk each): every warp load reads two
        // whole 256-byte rows, so global reads stay coalesced
        const uint32_t base = smem_u32(smem + stage * kTileBytes);
        const size_t ld = static_cast<size_t>(p.Hkv) * 128;
        const int c = lane & 15;
#pragma unroll
        for (int i = 0; i < kTile / 2; ++i) {
          const int r = 2 * i + (lane >> 4);
          const int src = __shfl_sync(0xffffffffu, i < 16 ? i0 : i1, r & 31);
          const int64_t row = static_cast<int64_t>(src);
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
    // ------------------------------------------------------------ consumer warp
    const int G = p.Hq / p.Hkv;
    const int g = lane >> 2, t4 = lane & 3;
    const float sc = p.scale * kLog2e;
    int stage = 0;
    uint32_t phase = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      const Item x = item_of(p, it);
      // Q fragments: rows = heads of this kv group (zero padded to 16)
      uint32_t qf[8][4];
      {
        const __nv_bfloat16* q0 = p.q + static_cast<size_t>(x.b) * p.ldq + static_cast<size_t>(x.kvh * G + g) * 128;
        const __nv_bfloat16* q8 = q0 + 8 * 128;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int c = kk * 16 + t4 * 2;
          qf[kk][0] = g < G ? *reinterpret_cast<const uint32_t*>(q0 + c) : 0u;
          qf[kk][1] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(q8 + c) : 0u;
          qf[kk][2] = g < G ? *reinterpret_cast<const uint32_t*>(q0 + c + 8) : 0u;
          qf[kk][3] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(q8 + c + 8) : 0u;
        }
      }
      float o[16][4];
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
      bool ok = true;
      for (int t0 = x.k0; t0 < x.k1; t0 += kTile) {
        if (!mbar_wait(&full[stage], phase, abort_flag, status, 800 + stage)) {
          ok = false;
          break;
        }
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
            const int c = kk * 2 + ((lane >> 3) & 1);
            ldsm_x4(sK + tile_off(r, c), b0, b1, b2, b3);
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
            const int c = dp * 2 + (lane >> 4);
            ldsm_x4_t(sV + tile_off(r, c), b0, b1, b2, b3);
            mma_bf16(o[2 * dp], a0, a1, a2, a3, b0, b1);
            mma_bf16(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
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
      // write this item's result: rows g (and g+8) of the 16-row tile are heads kvh*G + row
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float l = lrow[hr];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        const int row = g + hr * 8;
        if (row < G) {
          const int hq = x.kvh * G + row;
          const float inv = l > 0.f ? 1.f / l : 0.f;
          if (p.num_splits == 1) {
            __nv_bfloat16* orow = p.o + static_cast<size_t>(x.b) * p.ldo + static_cast<size_t>(hq) * 128;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              *reinterpret_cast<uint32_t*>(orow + i * 8 + t4 * 2) =
                  pack_bf16x2(o[i][hr * 2] * inv, o[i][hr * 2 + 1] * inv);
          } else {
            const size_t base = (static_cast<size_t>(x.b) * p.Hq + hq) * p.num_splits + x.split;
            float* po = p.part_o + base * 128;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              *reinterpret_cast<float2*>(po + i * 8 + t4 * 2) = make_float2(o[i][hr * 2] * inv, o[i][hr * 2 + 1] * inv);
            if (t4 == 0) p.part_lse[base] = l > 0.f ? mrow[hr] + log2f(l) : -INFINITY;
          }
        }
      }
    }
  }
}

__global__ void decode_persistent_combine_kernel(DecodePersistParams p) {
  grid_dep_launch();
  const int b = blockIdx.x, hq = blockIdx.y;
  const size_t base = (static_cast<size_t>(b) * p.Hq + hq) * p.num_splits;
  float M = -INFINITY;
  for (int s = 0; s < p.num_splits; ++s) M = fmaxf(M, p.part_lse[base + s]);
  const float mref = M == -INFINITY ? 0.f : M;
  for (int c = threadIdx.x; c < 128; c += blockDim.x) {
    float L = 0.f, acc = 0.f;
    for (int s = 0; s < p.num_splits; ++s) {
      const float w = exp2f(p.part_lse[base + s] - mref);
      L += w;
      acc += w * p.part_o[(base + s) * 128 + c];
    }
    p.o[static_cast<size_t>(b) * p.ldo + static_cast<size_t>(hq) * 128 + c] =
        __float2bfloat16(L > 0.f ? acc / L : 0.f);
  }
}

int decode_persistent_smem_bytes() { return kStages * kTileBytes + 1024 + 2 * kStages * 8 + 16; }

void decode_persistent_launch(const DecodePersistParams& p, int grid, int* status, cudaStream_t st) {
  static SmemOptIn opt;
  opt.ensure(decode_persistent_kernel, decode_persistent_smem_bytes());
  decode_persistent_kernel<<<grid, 64, decode_persistent_smem_bytes(), st>>>(p, status);
  if (p.num_splits > 1) decode_persistent_combine_kernel<<<dim3(p.B, p.Hq), 128, 0, st>>>(p);
}

}  // namespace octo
