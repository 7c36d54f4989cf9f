// noalloc.cu — a W8A8 matmul entry point that allocates nothing.
//
// rb_matmul quantises the activation rows of a W8A8 call into engine-owned
// scratch that grows with cudaMalloc on first use of a larger shape. Some
// callers cannot allow that: code running while a CUDA graph is being
// captured (cudaMalloc is not stream-ordered and breaks the capture), callers
// that run under a fixed device-memory budget or a custom allocator, and
// real-time paths where a synchronising allocation is an unbounded stall.
// rb_matmul_w8a8_noalloc stages the same int8 codes and row scales in a
// file-scope device array instead, sized once at library load.
//
// Contract (also in include/rocket_b200.h):
//   * one shared array of kNoAllocScratchBytes per GPU that loads the library,
//     held until process exit; a call needs round_up(m*k, 256) + 4*m bytes
//     and is rejected with RB_E_SHAPE beyond that;
//   * the first call on a device resolves the array's device address
//     (cudaGetSymbolAddress) with that device current; make that first call
//     before any stream capture;
//   * every call overwrites the part of the array it uses and nothing needs
//     to start at zero (rows past m are never read); calls whose work
//     overlaps on the GPU (other streams, other host threads) race on the
//     array and must be serialised by the caller.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "kernels.h"

namespace rb {

// Maximum staging for one call: int8 codes [m, k] (256-byte aligned) plus f32
// row scales [m].
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device ordinal. In host code the
// array's name is only a host-side stand-in, so the address is resolved once
// per device (with that device current) and passed to the kernels.
static void* g_scratch_addr[64] = {};
static std::mutex g_scratch_mu;

static int noalloc_scratch(int device, void** out) {
  if (device < 0 || device >= 64) return report_error(RB_E_DEVICE, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      char msg[256];
      snprintf(msg, sizeof(msg), "cudaGetSymbolAddress(no-alloc scratch) failed: %s",
               cudaGetErrorString(e));
      return report_error(RB_E_DEVICE, msg);
    }
    g_scratch_addr[device] = p;
  }
  *out = g_scratch_addr[device];
  return RB_OK;
}

}  // namespace rb

using namespace rb;

extern "C" int rb_matmul_w8a8_noalloc(int64_t id, const void* x, int x_dtype, int64_t m, int64_t k,
                                      void* y, int y_dtype, void* stream) {
  if (!x || !y) return report_error(RB_E_SHAPE, "null matmul buffer");
  if (m <= 0) return report_error(RB_E_SHAPE, "matmul needs M > 0");
  if (x_dtype < RB_DTYPE_F32 || x_dtype > RB_DTYPE_BF16 || y_dtype < RB_DTYPE_F32 ||
      y_dtype > RB_DTYPE_BF16)
    return report_error(RB_E_SHAPE, "bad dtype");
  W8A8View v;
  int rc = w8a8_view(id, &v);  // also makes the engine's device current
  if (rc != RB_OK) return rc;
  if (k != v.k) return report_error(RB_E_SHAPE, "activation K mismatch for the W8A8 weight");
  if (v.act != RB_ACT_NONE && y_dtype != RB_DTYPE_F16)
    return report_error(RB_E_SHAPE, "the W8A8 weight has a fused activation: the output must be f16");
  // The same output contract as rb_matmul.
  const int64_t y_bytes = y_dtype == RB_DTYPE_F32 ? 4 : 2;
  if ((v.n * y_bytes) % 16 != 0 && (reinterpret_cast<uintptr_t>(y) & 15) != 0)
    return report_error(RB_E_SHAPE, "output buffer must be 16-byte aligned");
  const size_t codes_bytes = (static_cast<size_t>(m) * static_cast<size_t>(k) + 255) & ~size_t(255);
  const size_t need = codes_bytes + static_cast<size_t>(m) * sizeof(float);
  if (m > (int64_t(1) << 30) || need > kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "rb_matmul_w8a8_noalloc: m*k = %lld needs %zu bytes of staging, above the fixed "
             "%zu-byte no-allocation scratch; split the rows or use rb_matmul",
             static_cast<long long>(m) * static_cast<long long>(k), need, kNoAllocScratchBytes);
    return report_error(RB_E_SHAPE, msg);
  }
  void* base = nullptr;
  if ((rc = noalloc_scratch(v.device, &base)) != RB_OK) return rc;
  int8_t* codes = reinterpret_cast<int8_t*>(base);
  float* row_scale = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(base) + codes_bytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  if ((rc = launch_quantize_rows_i8(x, x_dtype, m, k, v.in_scale, codes, row_scale, st)) != RB_OK)
    return report_error(rc, "row quantiser launch failed");
  count_launches(1);
  CUtensorMap tmA, tmC;
  if ((rc = make_tmap_2d(&tmA, codes, 1, m, k, k, 128, 128, 128)) != RB_OK) return rc;
  GemmLaunch L{};
  L.M = static_cast<int>(m);
  L.N = static_cast<int>(v.n);
  L.K = static_cast<int>(v.k);
  L.s_row = row_scale;
  L.s_col = v.w_scale;
  L.out = y;
  L.ldo = static_cast<int>(v.n);
  L.out_dtype = y_dtype;
  L.out_scale = v.out_scale;
  L.act = v.act;
  L.err = v.err;
  L.num_sms = v.num_sms;
  L.pdl = 1;  // the GEMM's prologue overlaps the quantiser launched just before it
  const bool tstore = make_output_map(&tmC, y, y_dtype, m, v.n);
  const GemmPlan plan = gemm_plan(true, L.M, L.N, L.K, v.num_sms);
  if ((rc = launch_w8a8_gemm(L, plan, tmA, v.tm_codes[bn_index(plan.weight_rows())],
                             tstore ? &tmC : nullptr, st)) != RB_OK)
    return report_error(rc, "w8a8 gemm launch failed");
  count_launches(1);
  return RB_OK;
}
