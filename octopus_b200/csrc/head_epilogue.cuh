// GEMM epilogues that reduce a vocabulary tile instead of storing it.
//
// EpiHeadLse  (training logprob head): the accumulator tile holds logits
//   z = alpha * h . W_v   (alpha = 1/temperature) for 128 rows x BN vocab columns.
//   Each thread owns one row and emits, per (row, vocab tile), the partial
//     m = max z,  s = sum exp(z - m),  t = sum exp(z - m) * z,  zl = z[label] (0 if absent)
//   into partial[row, tile, 0..3].  A combine pass turns the partials into
//     lse = M + log S,  logp = z_label - lse,  entropy = lse - T / S.
//   Full logits never reach global memory.
//
// EpiSample   (rollout sampling head): same tile, emits
//     m, s (for the log-normaliser), the best Gumbel-perturbed score z + g and its column.
//   Gumbel-max over the whole vocabulary is an exact sample from softmax(z).
//   The noise is a counter-based hash of (seed, row stream, column), so a sample
//   does not depend on how rows are batched or how the vocabulary is tiled.
#pragma once
#include "common.cuh"

namespace octo {

// SplitMix64 finaliser (Steele, Lea & Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014): a bijective 64-bit mixer used as a counter-based RNG.
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// 32-bit integer mixer "lowbias32" (C. Wellons, hash-prospector, 2018; public domain
// construction: xorshift-multiply rounds).  Cheap enough to run once per logit.
__host__ __device__ __forceinline__ uint32_t lowbias32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

// Per-row key: computed once per (row, tile) from the 64-bit seed and row stream.
__device__ __forceinline__ uint32_t row_key(uint64_t seed, uint64_t stream) {
  return static_cast<uint32_t>(splitmix64(seed ^ splitmix64(stream)) >> 32);
}

// Uniform strictly inside (0, 1) from (row key, column): 23 high bits plus half a step,
// so u is in [2^-24, 1 - 2^-24], both exactly representable in fp32 (a 24-bit
// variate plus half a step would round its top value to exactly 1.0).
__device__ __forceinline__ float hash_uniform(uint32_t key, uint32_t col) {
  const uint32_t h = lowbias32(key ^ (col * 0x9E3779B9u));
  return (static_cast<float>(h >> 9) + 0.5f) * (1.0f / 8388608.0f);
}

// Standard Gumbel noise -log(-log u) (fast log intrinsics; sampling-grade accuracy).
__device__ __forceinline__ float gumbel_noise(uint32_t key, uint32_t col) {
  const float u = hash_uniform(key, col);
  return -__logf(-__logf(u));
}

struct EpiHeadLse {
  const int32_t* labels;
  float* partial;  // [M, n_tiles, 4]
  int n_tiles;
  int bn;
  float alpha;
  int vocab_limit;
  // per-thread running state for the current tile
  float m, s, t, zl;
  int label;

  __device__ __forceinline__ void begin_split(int) {}
  __device__ __forceinline__ void begin_tile() {
    m = -INFINITY;
    s = 0.f;
    t = 0.f;
    zl = 0.f;
    label = -1;
  }
  __device__ __forceinline__ void apply(int row, int col0, int nvalid, float (&v)[32], int) {
    if (label < 0) label = labels[row];
    float cm = -INFINITY;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      v[i] *= alpha;
      const bool ok = (i < nvalid) && (col0 + i < vocab_limit);
      if (!ok) v[i] = -INFINITY;
      cm = fmaxf(cm, v[i]);
      if (col0 + i == label) zl = v[i];
    }
    if (cm == -INFINITY) return;
    const float nm = fmaxf(m, cm);
    const float scale = (m == -INFINITY) ? 0.f : __expf(m - nm);
    float cs = 0.f, ct = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float e = (v[i] == -INFINITY) ? 0.f : __expf(v[i] - nm);
      cs += e;
      ct += e * ((v[i] == -INFINITY) ? 0.f : v[i]);
    }
    s = s * scale + cs;
    t = t * scale + ct;
    m = nm;
  }
  __device__ __forceinline__ void end_tile(int row, int nb) {
    float4 o = make_float4(m, s, t, zl);
    *reinterpret_cast<float4*>(partial + (static_cast<size_t>(row) * n_tiles + nb) * 4) = o;
  }
  __device__ __forceinline__ void finish() const {}
};

struct EpiSample {
  float* partial;  // [M, n_tiles, 4] = (m, s, best score, best col as int bits)
  int n_tiles;
  int bn;
  float alpha;
  int vocab_limit;
  uint64_t seed;
  const int64_t* row_stream;
  int col_base;    // global vocabulary index of local column 0 (vocab-parallel shards)
  float m, s, best;
  int best_col;
  uint32_t key;
  bool have_stream;

  __device__ __forceinline__ void begin_split(int) {}
  __device__ __forceinline__ void begin_tile() {
    m = -INFINITY;
    s = 0.f;
    best = -INFINITY;
    best_col = -1;
    have_stream = false;
  }
  __device__ __forceinline__ void apply(int row, int col0, int nvalid, float (&v)[32], int) {
    if (!have_stream) {
      const uint64_t stream =
          row_stream != nullptr ? static_cast<uint64_t>(row_stream[row]) : static_cast<uint64_t>(row);
      key = row_key(seed, stream);
      have_stream = true;
    }
    float cm = -INFINITY;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      v[i] *= alpha;
      const bool ok = (i < nvalid) && (col0 + i < vocab_limit);
      if (!ok) v[i] = -INFINITY;
      cm = fmaxf(cm, v[i]);
    }
    if (cm == -INFINITY) return;
    const float nm = fmaxf(m, cm);
    const float scale = (m == -INFINITY) ? 0.f : __expf(m - nm);
    float cs = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (v[i] != -INFINITY) {
        cs += __expf(v[i] - nm);
        const float g = v[i] + gumbel_noise(key, static_cast<uint32_t>(col_base + col0 + i));
        if (g > best) {
          best = g;
          best_col = col_base + col0 + i;
        }
      }
    }
    s = s * scale + cs;
    m = nm;
  }
  __device__ __forceinline__ void end_tile(int row, int nb) {
    float4 o = make_float4(m, s, best, __int_as_float(best_col));
    *reinterpret_cast<float4*>(partial + (static_cast<size_t>(row) * n_tiles + nb) * 4) = o;
  }
  __device__ __forceinline__ void finish() const {}
};

}  // namespace octo

namespace octo {

// Backward of the logprob head, fused into the recompute GEMM: for each logit z
// (z = alpha * acc) with p = exp(z - lse) and logp = z - lse,
//   d logp_label / dz = onehot - p
//   d entropy / dz    = -p * (logp + H)
// so  dacc = alpha * ( g_lp * (onehot - p) - g_H * p * (logp + H) ),
// written as bf16 into C (row stride ldc).  Padded vocabulary columns get 0.
struct EpiHeadGrad {
  __nv_bfloat16* C;
  int ldc;
  const int32_t* labels;
  const float* lse;
  const float* ent;
  const float* g_lp;
  const float* g_ent;
  float alpha;
  int vocab_limit;
  __device__ __forceinline__ void begin_split(int) {}
  __device__ __forceinline__ void begin_tile() {}
  __device__ __forceinline__ void apply(int row, int col0, int nvalid, float (&v)[32], int) {
    const int lab = labels[row];
    const float L = lse[row], H = ent[row], gl = g_lp[row], gh = g_ent[row];
    __nv_bfloat16* dst = C + static_cast<size_t>(row) * ldc + col0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int col = col0 + i;
      float d = 0.f;
      if (col < vocab_limit) {
        const float lp = alpha * v[i] - L;
        const float p = __expf(lp);
        d = gl * ((col == lab ? 1.f : 0.f) - p) - gh * p * (lp + H);
        d *= alpha;
      }
      v[i] = d;
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
  __device__ __forceinline__ void end_tile(int, int) {}
  __device__ __forceinline__ void finish() const {}
};

}  // namespace octo
