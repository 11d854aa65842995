// Tensor-parallel fused kernels over NVLink peer memory (sm_100a).
//
//   AG -> GEMM   the persistent tcgen05 GEMM with an A source that gathers the
//                sequence-sharded activation into a LOCAL staging buffer: the epilogue
//                warps copy each remote row over NVLink once with plain 16-byte peer loads
//                (after a bounded wait for the owner's "shard ready" signal) and publish
//                per-128-row-block readiness counters, while the producer starts on the
//                rank's own rows.  The producer's TMA loads read local memory only (the
//                rank's own shard or the staging buffer, after the block's counter is
//                complete), so the transfer overlaps the MMAs block by block.
//   GEMM -> RS   the same GEMM with an epilogue that stores each accumulator row as bf16
//                into the receive buffer of the rank owning that row (peer stores), then
//                signals; the owner's reduce kernel sums the tp partials in rank order
//                with the residual and applies the next RMSNorm.
//   sampling     vocab-parallel Gumbel-max: per-rank partials of the sampling GEMM are
//                combined locally, exchanged (4 floats per row) by peer stores, merged.
//   barrier      single-CTA bounded barrier on a counter slot.
//   reshard      strided 2D copies from the trainer's weight layout to TP shards.
//
// All waits are bounded (status word budget, default OCTO_WAIT_NS); a timeout records kErrPeerTimeout in the
// status word, raises the CTA abort flag and returns without touching peer data.
#include <cuda_bf16.h>

#include "common.cuh"
#include "gemm_sm100.cuh"
#include "head_epilogue.cuh"
#include "tp.h"

namespace octo {

namespace {

__device__ __forceinline__ void red_release_sys_add(int* p, int v) {
  asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ bool wait_ge(const int* f, int target, volatile int* abort, int* status, int where) {
  const uint64_t t0 = globaltimer_ns();
  const uint64_t budget = wait_budget_ns(status);
  while (ld_acquire_sys(f) < target) {
    if (abort != nullptr && *abort) return false;
    if (globaltimer_ns() - t0 > budget) {
      record_error(status, kErrPeerTimeout, where);
      if (abort != nullptr) *abort = 1;
      return false;
    }
    __nanosleep(100);
  }
  return true;
}

__device__ __forceinline__ void signal_peers(const TpSlot& s) {
  __threadfence_system();
  for (int r = 0; r < s.tp; ++r)
    if (r != s.me) red_release_sys_add(s.peer_flags[r] + s.me, 1);
}

// Last CTA of the waiting kernel: consume one call's worth of every peer's signals.
__device__ __forceinline__ void consume(const TpSlot& s, int per_call) {
  if (atomicAdd(s.done, 1) == static_cast<int>(gridDim.x) - 1) {
    atomicExch(s.done, 0);
    for (int r = 0; r < s.tp; ++r)
      if (r != s.me) atomicAdd_system(s.flags + r, -per_call);
  }
}

__device__ bool wait_peers(const TpSlot& s, int target, int* status, int where) {
  for (int r = 0; r < s.tp; ++r) {
    if (r == s.me) continue;
    if (!wait_ge(s.flags + r, target, nullptr, status, where + r)) return false;
  }
  return true;
}

}  // namespace

// ---------------------------------------------------------------- AG -> GEMM A source
constexpr int kChunkRows = 2;  // staging copy granularity (rows of one peer shard)

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct AGather {
  CUtensorMap m[kMaxTp];
  const __nv_bfloat16* peer_x[kMaxTp];
  __nv_bfloat16* stage;
  int* work;
  int ldx, K, M, m_tiles;
  int rows_s, box_rows;
  TpSlot slot;
  int peer_grid;

  __device__ __forceinline__ void prefetch() const {
    for (int r = 0; r < slot.tp; ++r) tma_prefetch_desc(&m[r]);
  }
  __device__ __forceinline__ void signal() const { signal_peers(slot); }
  // remote rows of M-block mb, in chunks
  __device__ __forceinline__ int remote_chunks(int mb) const {
    const int g0 = mb * kGemmBM, g1 = min(M, g0 + kGemmBM);
    const int o0 = max(g0, slot.me * rows_s), o1 = min(g1, (slot.me + 1) * rows_s);
    return ((g1 - g0) - max(0, o1 - o0)) / kChunkRows;
  }
  // Epilogue warps of every CTA: copy peer chunks into the staging buffer until the work
  // counter runs out (so the copy never depends on which CTAs are resident).
  __device__ void prologue(int t, volatile int* abort, int* status) const {
    const int per_rank = rows_s / kChunkRows;
    const int total = (slot.tp - 1) * per_rank;
    const int cpr = K / 8;                       // 16-byte pieces per row
    __shared__ int chunk;
    uint32_t seen = 0;
    for (;;) {
      if (t == 0) chunk = atomicAdd(work, 1);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int c = chunk;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (c >= total) break;
      const int ri = c / per_rank;
      const int r = ri < slot.me ? ri : ri + 1;
      const int l0 = (c - ri * per_rank) * kChunkRows;
      if (!((seen >> r) & 1u)) {
        // the peer's shard is complete once any of its CTAs has signalled this call
        if (t == 0 && !wait_ge(slot.flags + r, 1, abort, status, 950 + r)) chunk = -1;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (chunk < 0) return;
        seen |= 1u << r;
      }
      const __nv_bfloat16* src = peer_x[r] + static_cast<size_t>(l0) * ldx;
      __nv_bfloat16* dst = stage + (static_cast<size_t>(r) * rows_s + l0) * K;
      // all loads of the chunk in flight before any store (one NVLink round trip per 8 pieces)
      constexpr int kPer = 8;
      for (int p0 = t; p0 < kChunkRows * cpr; p0 += 128 * kPer) {
        uint4 buf[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
          const int p = p0 + u * 128;
          if (p < kChunkRows * cpr) {
            const int row = p / cpr, col = (p - row * cpr) * 8;
            buf[u] = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(row) * ldx + col);
          }
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
          const int p = p0 + u * 128;
          if (p < kChunkRows * cpr) {
            const int row = p / cpr, col = (p - row * cpr) * 8;
            *reinterpret_cast<uint4*>(dst + static_cast<size_t>(row) * K + col) = buf[u];
          }
        }
      }
      fence_proxy_async_global();  // generic-proxy stores -> the producers' TMA reads
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (t == 0) red_release_gpu_add(work + 1 + (r * rows_s + l0) / kGemmBM, 1);
    }
  }
  __device__ bool ready(int mb, uint32_t&, volatile int* abort, int* status) const {
    const int need = remote_chunks(mb);
    if (need == 0) return true;
    const uint64_t t0 = globaltimer_ns();
    const uint64_t budget = wait_budget_ns(status);
    while (ld_acquire_gpu(work + 1 + mb) < need) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > budget) {
        record_error(status, kErrPeerTimeout, 940);
        *abort = 1;
        return false;
      }
      __nanosleep(64);
    }
    fence_proxy_async_global();
    return true;
  }
  // Last CTA: reset the staging counters and consume the peers' signals of this call.
  __device__ __forceinline__ void finish_cta() const {
    if (atomicAdd(slot.done, 1) == static_cast<int>(gridDim.x) - 1) {
      for (int i = 0; i <= m_tiles; ++i) work[i] = 0;
      __threadfence();
      atomicExch(slot.done, 0);
      for (int r = 0; r < slot.tp; ++r)
        if (r != slot.me) atomicAdd_system(slot.flags + r, -peer_grid);
    }
  }
  // ranks whose rows make up M-block mb: [r0, r1)
  __device__ __forceinline__ void ranks(int mb, int& r0, int& r1) const {
    if (rows_s >= kGemmBM) {
      r0 = (mb * kGemmBM) / rows_s;
      r1 = r0 + 1;
    } else {
      const int segs = kGemmBM / rows_s;
      r0 = mb * segs;
      r1 = min(slot.tp, r0 + segs);
    }
  }
  __device__ __forceinline__ uint32_t bytes(int mb) const {
    int r0, r1;
    ranks(mb, r0, r1);
    return static_cast<uint32_t>((r1 - r0) * box_rows * kGemmBK * 2);
  }
  __device__ __forceinline__ void load(uint8_t* dst, uint64_t* bar, int k0, int mb) const {
    if (rows_s >= kGemmBM) {
      const int r = (mb * kGemmBM) / rows_s;
      tma_load_2d(dst, &m[r], bar, k0, mb * kGemmBM - r * rows_s);
    } else {
      int r0, r1;
      ranks(mb, r0, r1);
      // box_rows is a multiple of 8: every segment starts on a 1024-byte swizzle atom
      for (int r = r0; r < r1; ++r) tma_load_2d(dst + (r - r0) * box_rows * 128, &m[r], bar, k0, 0);
    }
  }
};

// ---------------------------------------------------------------- GEMM -> RS epilogue
struct EpiRS {
  __nv_bfloat16* dst[kMaxTp];
  int ldc, rows_s;
  TpSlot slot;
  int part;  // receive slot: split * tp + sending rank (split-K partials are summed by the owner)
  __device__ __forceinline__ void begin_split(int ks) { part = ks * slot.tp + slot.me; }
  __device__ __forceinline__ void begin_tile() {}
  __device__ __forceinline__ __nv_bfloat16* row_dst(int row, int col0) const {
    const int owner = row / rows_s;
    return dst[owner] + (static_cast<size_t>(part) * rows_s + (row - owner * rows_s)) * ldc + col0;
  }
  __device__ __forceinline__ void apply(int row, int col0, int nvalid, float (&v)[32], int) {
    uint4 o[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      o[g].x = pack_bf16x2(v[g * 8 + 0], v[g * 8 + 1]);
      o[g].y = pack_bf16x2(v[g * 8 + 2], v[g * 8 + 3]);
      o[g].z = pack_bf16x2(v[g * 8 + 4], v[g * 8 + 5]);
      o[g].w = pack_bf16x2(v[g * 8 + 6], v[g * 8 + 7]);
    }
    const int lane = threadIdx.x & 31;
    if (__activemask() == 0xffffffffu && __all_sync(0xffffffffu, nvalid == 32)) {
      // a warp's 32 rows x 32 columns go through shared memory so each store instruction
      // writes 8 rows x 64 contiguous bytes (peer writes travel in larger NVLink packets)
      __shared__ uint4 stile[4][32][4];
      const int w = (threadIdx.x >> 5) & 3;
#pragma unroll
      for (int g = 0; g < 4; ++g) stile[w][lane][g] = o[g];
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int rl = it * 8 + (lane >> 2), piece = lane & 3;
        const int r = __shfl_sync(0xffffffffu, row, rl);
        *reinterpret_cast<uint4*>(row_dst(r, col0) + piece * 8) = stile[w][rl][piece];
      }
      __syncwarp();
      return;
    }
    __nv_bfloat16* out = row_dst(row, col0);
#pragma unroll
    for (int g = 0; g < 4; ++g)
      if (g * 8 < nvalid) *reinterpret_cast<uint4*>(out + g * 8) = o[g];
  }
  __device__ __forceinline__ void end_tile(int, int) {}
  __device__ __forceinline__ void finish() {
    // every epilogue thread's stores are ordered before the CTA's one signal
    __threadfence_system();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (threadIdx.x == 64) signal_peers(slot);
  }
};

template <int BN, class Epi, class ASrc>
static void launch_tp(const GemmLaunch& g, const Epi& epi, const ASrc& a) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_tcgen05_kernel<BN, false, false, Epi, ASrc>;
  static SmemOptIn opt;
  opt.ensure(kern, Cfg::kSmemBytes);
  kern<<<g.grid, kGemmThreads, Cfg::kSmemBytes, g.stream>>>(a, g.tb, g.s, epi, g.status);
}

void ag_gemm_launch(const AgLaunch& L) {
  const GemmLaunch& g = L.g;
  AGather a;
  for (int r = 0; r < kMaxTp; ++r) {
    a.m[r] = L.a[r];
    a.peer_x[r] = static_cast<const __nv_bfloat16*>(L.peer_x[r]);
  }
  a.stage = static_cast<__nv_bfloat16*>(L.stage);
  a.work = L.work;
  a.ldx = L.ldx;
  a.K = g.s.K;
  a.M = g.s.M;
  a.m_tiles = g.s.m_tiles;
  a.rows_s = L.rows_s;
  a.box_rows = L.box_rows;
  a.slot = L.slot;
  a.peer_grid = L.peer_grid;
  EpiBF16 e{reinterpret_cast<__nv_bfloat16*>(g.C), g.ldc, reinterpret_cast<const __nv_bfloat16*>(g.R), g.ldr,
            g.alpha, reinterpret_cast<const __nv_bfloat16*>(g.bias)};
  if (g.epi == kEpiSplitK) {
    EpiSplitK es{reinterpret_cast<float*>(g.C), g.s.M, g.s.N, nullptr};
    if (g.bn == 256) launch_tp<256>(g, es, a);
    else if (g.bn == 128) launch_tp<128>(g, es, a);
    else launch_tp<64>(g, es, a);
    return;
  }
  if (g.epi == kEpiSample) {
    EpiSample es{g.partial, g.s.n_tiles, g.bn, g.alpha, g.vocab_limit, g.seed, g.row_offset, g.col_base};
    if (g.bn == 256) launch_tp<256>(g, es, a);
    else if (g.bn == 128) launch_tp<128>(g, es, a);
    else launch_tp<64>(g, es, a);
    return;
  }
  if (g.bn == 256) launch_tp<256>(g, e, a);
  else if (g.bn == 128) launch_tp<128>(g, e, a);
  else launch_tp<64>(g, e, a);
}

void gemm_rs_launch(const RsLaunch& L) {
  const GemmLaunch& g = L.g;
  EpiRS e;
  for (int r = 0; r < kMaxTp; ++r) e.dst[r] = reinterpret_cast<__nv_bfloat16*>(L.recv[r]);
  e.ldc = L.ldc;
  e.rows_s = L.rows_s;
  e.slot = L.slot;
  e.part = L.slot.me;
  ALocal<false> a{g.ta};
  if (g.bn == 256) launch_tp<256>(g, e, a);
  else if (g.bn == 128) launch_tp<128>(g, e, a);
  else launch_tp<64>(g, e, a);
}

// ---------------------------------------------------------------- reduce (+ RMSNorm)
__global__ void tp_reduce_kernel(const __nv_bfloat16* __restrict__ recv, int parts, __nv_bfloat16* h, int ldh,
                                 int N, int rows_s, const __nv_bfloat16* __restrict__ w, __nv_bfloat16* x, int ldx,
                                 float eps, int plus_one, TpSlot slot, int peer_grid, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_peers(slot, peer_grid, status, 960) ? 1 : 0;
  __syncthreads();
  const int warps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (ok) {
    for (int row = blockIdx.x * warps + warp; row < rows_s; row += gridDim.x * warps) {
      __nv_bfloat16* hr = h + static_cast<size_t>(row) * ldh;
      float ss = 0.f;
      for (int c = lane * 8; c < N; c += 256) {
        float a[8];
        load8(hr + c, a);
        for (int r = 0; r < parts; ++r) {
          float b[8];
          load8(recv + (static_cast<size_t>(r) * rows_s + row) * N + c, b);
#pragma unroll
          for (int i = 0; i < 8; ++i) a[i] += b[i];
        }
        uint4 o;
        o.x = pack_bf16x2(a[0], a[1]);
        o.y = pack_bf16x2(a[2], a[3]);
        o.z = pack_bf16x2(a[4], a[5]);
        o.w = pack_bf16x2(a[6], a[7]);
        *reinterpret_cast<uint4*>(hr + c) = o;
        float q[8];
        load8(hr + c, q);  // rounded values (the norm sees what the next layer reads)
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += q[i] * q[i];
      }
      if (x == nullptr) continue;
      ss = warp_sum(ss);
      const float rstd = rsqrtf(ss / static_cast<float>(N) + eps);
      __nv_bfloat16* xr = x + static_cast<size_t>(row) * ldx;
      for (int c = lane * 8; c < N; c += 256) {
        float a[8], ww[8];
        load8(hr + c, a);
        load8(w + c, ww);
        float y[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = a[i] * rstd * (plus_one ? 1.f + ww[i] : ww[i]);
        uint4 o;
        o.x = pack_bf16x2(y[0], y[1]);
        o.y = pack_bf16x2(y[2], y[3]);
        o.z = pack_bf16x2(y[4], y[5]);
        o.w = pack_bf16x2(y[6], y[7]);
        *reinterpret_cast<uint4*>(xr + c) = o;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) consume(slot, peer_grid);
}

int tp_reduce(const void* recv, int parts, void* h, int ldh, int N, int rows_s, const void* w, void* x, int ldx,
              float eps, int plus_one, const TpSlot& slot, int peer_grid, int* status, cudaStream_t st) {
  const int grid = max(1, min((rows_s + 7) / 8, 148 * 4));
  tp_reduce_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(recv), parts,
                                         static_cast<__nv_bfloat16*>(h),
                                         ldh, N, rows_s, static_cast<const __nv_bfloat16*>(w),
                                         static_cast<__nv_bfloat16*>(x), ldx, eps, plus_one, slot, peer_grid, status);
  return grid;
}

// ---------------------------------------------------------------- vocab-parallel sampling
struct XchPtrs {
  float4* p[kMaxTp];
};

__global__ void tp_sample_local_kernel(const float* __restrict__ part, int M, int T, XchPtrs xch, TpSlot slot) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row < M) {
    const float4* p = reinterpret_cast<const float4*>(part) + static_cast<size_t>(row) * T;
    float gm = -INFINITY, best = -INFINITY;
    int best_col = -1;
    for (int i = lane; i < T; i += 32) {
      const float4 q = p[i];
      gm = fmaxf(gm, q.x);
      const int c = __float_as_int(q.w);
      if (c >= 0 && (q.z > best || (q.z == best && c < best_col) || best_col < 0)) {
        best = q.z;
        best_col = c;
      }
    }
    gm = warp_max(gm);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oc = __shfl_xor_sync(0xffffffffu, best_col, o);
      if (oc >= 0 && (ob > best || (ob == best && oc < best_col) || best_col < 0)) {
        best = ob;
        best_col = oc;
      }
    }
    float S = 0.f;
    for (int i = lane; i < T; i += 32) {
      const float4 q = p[i];
      if (q.x != -INFINITY) S += q.y * __expf(q.x - gm);
    }
    S = warp_sum(S);
    if (lane < slot.tp) {
      const float4 v = make_float4(gm, S, best, __int_as_float(best_col));
      xch.p[lane][static_cast<size_t>(slot.me) * M + row] = v;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) signal_peers(slot);
}

__global__ void tp_sample_final_kernel(const float4* __restrict__ xch, int M, uint64_t seed,
                                       const int64_t* __restrict__ row_stream, int64_t* tokens, float* logprob,
                                       TpSlot slot, int peer_grid, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_peers(slot, peer_grid, status, 970) ? 1 : 0;
  __syncthreads();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (ok && row < M) {
    float GM = -INFINITY, best = -INFINITY;
    int col = -1;
    for (int r = 0; r < slot.tp; ++r) {
      const float4 q = xch[static_cast<size_t>(r) * M + row];
      GM = fmaxf(GM, q.x);
      const int c = __float_as_int(q.w);
      if (c >= 0 && (q.z > best || (q.z == best && c < col) || col < 0)) {
        best = q.z;
        col = c;
      }
    }
    float S = 0.f;
    for (int r = 0; r < slot.tp; ++r) {
      const float4 q = xch[static_cast<size_t>(r) * M + row];
      if (q.x != -INFINITY) S += q.y * __expf(q.x - GM);
    }
    const uint64_t stream = row_stream != nullptr ? static_cast<uint64_t>(row_stream[row]) : static_cast<uint64_t>(row);
    const float z = best - gumbel_noise(row_key(seed, stream), static_cast<uint32_t>(col));
    tokens[row] = col;
    logprob[row] = z - (GM + logf(S));
  }
  __syncthreads();
  if (threadIdx.x == 0) consume(slot, peer_grid);
}

int tp_sample_local(const float* part, int M, int T, void* const* xch, const TpSlot& slot, cudaStream_t st) {
  XchPtrs x{};
  for (int r = 0; r < slot.tp; ++r) x.p[r] = static_cast<float4*>(xch[r]);
  const int grid = max(1, (M + 7) / 8);
  tp_sample_local_kernel<<<grid, 256, 0, st>>>(part, M, T, x, slot);
  return grid;
}

void tp_sample_final(const void* xch_local, int M, uint64_t seed, const int64_t* row_stream, int64_t* tokens,
                     float* logprob, const TpSlot& slot, int peer_grid, int* status, cudaStream_t st) {
  tp_sample_final_kernel<<<max(1, (M + 127) / 128), 128, 0, st>>>(static_cast<const float4*>(xch_local), M, seed,
                                                                   row_stream, tokens, logprob, slot, peer_grid,
                                                                   status);
}

// ---------------------------------------------------------------- barrier
__global__ void tp_barrier_kernel(TpSlot slot, int* status) {
  if (threadIdx.x == 0) {
    signal_peers(slot);
    wait_peers(slot, 1, status, 980);
    for (int r = 0; r < slot.tp; ++r)
      if (r != slot.me) atomicAdd_system(slot.flags + r, -1);
    __threadfence_system();
  }
}

void tp_barrier(const TpSlot& slot, int* status, cudaStream_t st) {
  tp_barrier_kernel<<<1, 32, 0, st>>>(slot, status);
}

// ---------------------------------------------------------------- reshard copy
__global__ void reshard_copy_kernel(const ReshardSeg* __restrict__ segs, int nseg, int64_t total) {
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int lo = 0, hi = nseg - 1;
    while (lo < hi) {  // last segment with first <= c
      const int mid = (lo + hi + 1) >> 1;
      if (segs[mid].first <= c) lo = mid;
      else hi = mid - 1;
    }
    const ReshardSeg& s = segs[lo];
    const int64_t k = c - s.first;
    const int cpr = s.cols / 8;
    const int64_t row = k / cpr, col = (k - row * cpr) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(s.src) + row * s.lds + col);
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(s.dst) + row * s.ldd + col) = v;
  }
}

void reshard_copy(const ReshardSeg* segs, int nseg, int64_t total_chunks, cudaStream_t st) {
  if (total_chunks == 0 || nseg == 0) return;
  const int64_t want = (total_chunks + 255) / 256;
  const int grid = static_cast<int>(want < 148 * 8 ? want : 148 * 8);
  reshard_copy_kernel<<<grid, 256, 0, st>>>(segs, nseg, total_chunks);
}

}  // namespace octo
