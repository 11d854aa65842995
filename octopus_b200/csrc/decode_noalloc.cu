// Allocation-free variant of the split-K paged decode attention (see decode_noalloc.h for
// who needs it, its limits and its rules).  It has no counterpart in the reference
// project.
//
// The split-K partials live in file-scope device arrays of fixed size instead of a
// buffer from an allocator.  Host code cannot use the arrays' names as device
// addresses (in host code they name host-side stand-ins), so the first call on each
// device resolves their device addresses with cudaGetSymbolAddress while that device
// is current, and caches them per device.  The kernels are the regular decode kernels
// of attention.cu, launched through the same host launcher with these addresses as
// their scratch pointers.
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "attention.h"
#include "decode_noalloc.h"

static __device__ __align__(256) float g_noalloc_part_o[OCTO_NOALLOC_MAX_PARTIAL_FLOATS];
static __device__ __align__(256) float g_noalloc_part_lse[OCTO_NOALLOC_MAX_PARTIAL_ROWS];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_part_o_addr[kMaxDevices] = {nullptr};
float* g_part_lse_addr[kMaxDevices] = {nullptr};

// Resolve (once per device, with that device current) the device addresses of the
// scratch arrays.  Returns false if the runtime cannot resolve them.
bool scratch_addresses(int device, float** part_o, float** part_lse) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_part_o_addr[device] == nullptr) {
    void* a = nullptr;
    void* b = nullptr;
    cudaError_t e1 = cudaGetSymbolAddress(&a, g_noalloc_part_o);
    if (e1 != cudaSuccess || a == nullptr) {
      std::fprintf(stderr, "octo_decode_attention_noalloc: cudaGetSymbolAddress(part_o) failed on device %d: %s\n",
                   device, cudaGetErrorString(e1));
      return false;
    }
    cudaError_t e2 = cudaGetSymbolAddress(&b, g_noalloc_part_lse);
    if (e2 != cudaSuccess || b == nullptr) {
      std::fprintf(stderr, "octo_decode_attention_noalloc: cudaGetSymbolAddress(part_lse) failed on device %d: %s\n",
                   device, cudaGetErrorString(e2));
      return false;
    }
    g_part_o_addr[device] = static_cast<float*>(a);
    g_part_lse_addr[device] = static_cast<float*>(b);
  }
  *part_o = g_part_o_addr[device];
  *part_lse = g_part_lse_addr[device];
  return true;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int octo_decode_attention_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int32_t* kv_start, const int32_t* kv_len,
    const int32_t* kv_indices, void* o, int B, int Hq, int Hkv, int head_dim, int ldq, int ldo, int num_splits,
    float scale, cudaStream_t stream) {
  if (B <= 0) return OCTO_NOALLOC_OK;
  if ((head_dim != 64 && head_dim != 128) || Hkv <= 0 || Hq % Hkv != 0 || Hq / Hkv > 16 || num_splits < 1 ||
      num_splits > 64) {
    std::fprintf(stderr,
                 "octo_decode_attention_noalloc: unsupported shape (head_dim %d, Hq %d, Hkv %d, num_splits %d); "
                 "need head_dim 64 or 128, Hq %% Hkv == 0, Hq / Hkv <= 16, 1 <= num_splits <= 64\n",
                 head_dim, Hq, Hkv, num_splits);
    return OCTO_NOALLOC_ERR_UNSUPPORTED;
  }
  const long long rows = static_cast<long long>(B) * Hq * num_splits;
  const long long floats = rows * head_dim;
  if (num_splits > 1 && (floats > OCTO_NOALLOC_MAX_PARTIAL_FLOATS || rows > OCTO_NOALLOC_MAX_PARTIAL_ROWS)) {
    std::fprintf(stderr,
                 "octo_decode_attention_noalloc: B * Hq * num_splits * head_dim = %lld floats (limit %d) and "
                 "B * Hq * num_splits = %lld rows (limit %d) exceed the static scratch; lower the batch or "
                 "num_splits\n",
                 floats, OCTO_NOALLOC_MAX_PARTIAL_FLOATS, rows, OCTO_NOALLOC_MAX_PARTIAL_ROWS);
    return OCTO_NOALLOC_ERR_TOO_LARGE;
  }
  // The kernel reads K/V rows with 16-byte copies and q / writes o two bf16 at a time:
  // misaligned pointers or strides would fault on the GPU, so they are refused here.
  const auto addr = [](const void* p) { return reinterpret_cast<uintptr_t>(p); };
  const int row = Hq * head_dim;
  if ((addr(k_cache) | addr(v_cache)) % 16 != 0 || (addr(q) | addr(o)) % 4 != 0 ||
      (addr(kv_start) | addr(kv_len) | addr(kv_indices)) % 4 != 0 || ldq < row || ldo < row || ldq % 2 != 0 ||
      ldo % 2 != 0 || q == nullptr || o == nullptr || k_cache == nullptr || v_cache == nullptr ||
      kv_start == nullptr || kv_len == nullptr || kv_indices == nullptr) {
    std::fprintf(stderr,
                 "octo_decode_attention_noalloc: bad pointers or strides (k/v caches must be 16-byte aligned, q, o "
                 "and the int32 tables 4-byte aligned and non-null, ldq / ldo even and >= Hq * head_dim = %d; got "
                 "ldq %d, ldo %d)\n",
                 row, ldq, ldo);
    return OCTO_NOALLOC_ERR_UNSUPPORTED;
  }
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return OCTO_NOALLOC_ERR_SETUP;
  float* part_o = nullptr;
  float* part_lse = nullptr;
  if (num_splits > 1 && !scratch_addresses(device, &part_o, &part_lse)) return OCTO_NOALLOC_ERR_SETUP;

  octo::DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k_cache = static_cast<const __nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<const __nv_bfloat16*>(v_cache);
  p.o = static_cast<__nv_bfloat16*>(o);
  p.kv_start = kv_start;
  p.kv_len = kv_len;
  p.kv_indices = kv_indices;
  p.part_o = part_o;
  p.part_lse = part_lse;
  p.ldq = ldq;
  p.ldk = Hkv * head_dim;
  p.ldo = ldo;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.num_splits = num_splits;
  p.scale = scale;
  // the launcher returns the error of its own launches only (an unrelated pending error is
  // left for its owner to see)
  const cudaError_t e = octo::attn_decode(p, B, head_dim, stream);
  if (e != cudaSuccess) {
    std::fprintf(stderr, "octo_decode_attention_noalloc: launch failed: %s\n", cudaGetErrorString(e));
    return OCTO_NOALLOC_ERR_LAUNCH;
  }
  return OCTO_NOALLOC_OK;
}
