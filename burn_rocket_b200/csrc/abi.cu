// abi.cu — the extern "C" surface of librocket_b200.so (include/rocket_b200.h).
//
// Mirrors the engine of crates/burn-rocket/src/ext.rs: one global engine per
// process behind a mutex (ext.rs:537-556), a registry of resident weights with
// monotonically increasing ids (ext.rs:39-50, 829-840), and op entry points
// that validate shapes and report the reference's status codes. The device
// work itself lives in gemm.cu, quant.cu and attention.cu.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "kernels.h"
#include "sm100.cuh"

namespace rb {

// ------------------------------------------------------------------ errors
static thread_local std::string g_last_error;

static int fail(int rc, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return rc;
}

#define RB_CUDA(call, what)                                                                  \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      return fail(RB_E_DEVICE, "%s: %s (%s)", what, cudaGetErrorName(e_), cudaGetErrorString(e_)); \
  } while (0)

// ------------------------------------------------------------------ tensor maps
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static bool load_encode_fn() {
  if (g_encode) return true;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                       &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || fn == nullptr)
    return false;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return true;
}

int make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_stride_elems, uint32_t box_cols, uint32_t box_rows,
                 int swizzle_bytes) {
  if (!load_encode_fn()) return fail(RB_E_DEVICE, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return fail(RB_E_SHAPE, "tensor base %p is not 16-byte aligned", base);
  if ((row_stride_elems * elem_bytes) % 16 != 0)
    return fail(RB_E_SHAPE, "row stride %llu elements is not a multiple of 16 bytes",
                (unsigned long long)row_stride_elems);
  CUtensorMapDataType dt = elem_bytes == 1   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                           : elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                             : CU_TENSOR_MAP_DATA_TYPE_UINT32;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                        : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                        : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                              : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(RB_E_DEVICE, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu box=%ux%u",
                (int)r, (unsigned long long)rows, (unsigned long long)cols, box_cols, box_rows);
  return RB_OK;
}

// [rows, heads, d] view of head-strided f16 rows (dims: column in the head,
// head, row): a box of box_d columns of one head reads the elements past d as
// zeros, which stages a head narrower than the UMMA K granularity without a
// padded copy.
int make_tmap_heads(CUtensorMap* map, const void* base, uint64_t rows, uint64_t heads, uint64_t d,
                    uint64_t row_stride_elems, uint32_t box_d, uint32_t box_rows, int swizzle_bytes) {
  if (!load_encode_fn()) return fail(RB_E_DEVICE, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return fail(RB_E_SHAPE, "tensor base %p is not 16-byte aligned", base);
  if ((row_stride_elems * 2) % 16 != 0 || (d * 2) % 16 != 0)
    return fail(RB_E_SHAPE, "head rows: strides must be multiples of 16 bytes");
  cuuint64_t dims[3] = {d, heads, rows};
  cuuint64_t strides[2] = {d * 2, row_stride_elems * 2};
  cuuint32_t box[3] = {box_d, 1, box_rows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(RB_E_DEVICE, "cuTensorMapEncodeTiled (heads) failed (%d) rows=%llu heads=%llu d=%llu", (int)r,
                (unsigned long long)rows, (unsigned long long)heads, (unsigned long long)d);
  return RB_OK;
}

int bn_index(int bn) {
  switch (bn) {
    case 256: return 0;
    case 128: return 1;
    case 96: return 2;
    case 64: return 3;
    default: return -1;
  }
}

// ------------------------------------------------------------------ engine
struct Weight {
  int kind = 0;
  int64_t n = 0, k = 0;
  int8_t* codes = nullptr;   // [n, k]
  void* scales = nullptr;    // Q8_0: f16 [k/32, pitch]; W8A8: f32 [n]
  int64_t pitch = 0;         // Q8_0 scale row pitch: round_up(n, 8)
  float in_scale = 0.0f, out_scale = 0.0f;
  int64_t group = 0;         // RB_WEIGHT_I8G: K group width (scales f32 [n, k/group])
  float* scales_t = nullptr; // RB_WEIGHT_I8G: the scales group-major [k/group, ldb], zero past n
  int64_t ldb = 0;           // RB_WEIGHT_I8G: round_up(n, 128)
  bool gated = false;        // gate|up interleaved in 32-row blocks: matmul gives silu(gate)*up, n/2 columns
  int act = RB_ACT_NONE;     // element-wise activation fused into the matmul epilogue
  // TMA maps per staged weight-tile height ({256, 128, 96, 64}, see
  // bn_index; a CTA-pair tile stages half its N per CTA): the codes
  // (Q8_0: box 64 x bn; W8A8: box 128 x bn, 128-B swizzle) and the Q8_0
  // scales (box bn x 2).
  CUtensorMap tm_codes[4]{};
  CUtensorMap tm_scales[4]{};
  size_t bytes = 0;
};

// Builds the per-N-tile TMA maps of a packed weight.
static int weight_maps(Weight& w) {
  static const int bns[4] = {256, 128, 96, 64};
  for (int i = 0; i < 4; ++i) {
    const int bn = bns[i];
    int rc;
    if (w.kind == RB_WEIGHT_Q8_0) {
      if ((rc = make_tmap_2d(&w.tm_codes[i], w.codes, 1, w.n, w.k, w.k, 64, bn, 0)) != RB_OK) return rc;
      if ((rc = make_tmap_2d(&w.tm_scales[i], w.scales, 2, w.k / 32, w.n, w.pitch, bn, 2, 0)) != RB_OK)
        return rc;
    } else if (w.kind == RB_WEIGHT_F16) {
      if ((rc = make_tmap_2d(&w.tm_codes[i], w.codes, 2, w.n, w.k, w.k, 64, bn, 128)) != RB_OK) return rc;
    } else {
      if ((rc = make_tmap_2d(&w.tm_codes[i], w.codes, 1, w.n, w.k, w.k, 128, bn, 128)) != RB_OK) return rc;
    }
  }
  return RB_OK;
}

// Output map for the TMA-store epilogue, or false when the output pitch or
// base alignment rules it out (the kernel then stores directly).
static bool output_map(CUtensorMap* map, void* y, int y_dtype, int64_t m, int64_t n) {
  const int eb = (y_dtype == RB_DTYPE_F16 || y_dtype == RB_DTYPE_BF16) ? 2 : 4;
  if ((reinterpret_cast<uintptr_t>(y) & 15) != 0 || (n * eb) % 16 != 0) return false;
  const std::string saved = g_last_error;
  const bool ok = make_tmap_2d(map, y, eb, m, n, n, 128 / eb, 32, 128) == RB_OK;
  g_last_error = saved;
  return ok;
}

// Query-row chunks of the pipelined host-entry attention (rb_attention_host).
constexpr int kHostAttnChunks = 4;

struct Scratch {
  void* ptr = nullptr;
  size_t bytes = 0;
  int grow(size_t need, const char* what) {
    if (need <= bytes) return RB_OK;
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
    size_t want = need + need / 4 + 256;
    if (cudaMalloc(&ptr, want) != cudaSuccess) {
      cudaGetLastError();
      return fail(RB_E_NOMEM, "%s: cudaMalloc(%zu) failed", what, want);
    }
    bytes = want;
    return RB_OK;
  }
};

struct Engine {
  int device = -1;
  int num_sms = 0;
  uint32_t* err = nullptr;  // device error word
  float* attn_rec = nullptr;  // attention split-mode records (kAttnRecBytes)
  int* attn_cnt = nullptr;    // attention split-mode arrival counters (kAttnCntBytes)
  std::unordered_map<int64_t, Weight> weights;
  int64_t next_id = 1;
  Scratch act;       // activation staging (f16 or int8 codes)
  Scratch rowscale;  // per-row scales
  Scratch io_in, io_out, io_k, io_v;  // host-entry staging
  cudaStream_t host_stream = nullptr;
  // Pipelined host-entry attention: copies in, kernels, copies out on three
  // streams, ordered by events (created on first use).
  cudaStream_t pipe_in = nullptr, pipe_out = nullptr;
  cudaEvent_t pipe_ev[2 * kHostAttnChunks + 1] = {};
  bool pipe_ready = false;
};

static std::mutex g_mu;
static Engine* g_engine = nullptr;

static int ensure_pipe(Engine* e) {
  if (e->pipe_ready) return RB_OK;
  if (cudaStreamCreateWithFlags(&e->pipe_in, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&e->pipe_out, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    return fail(RB_E_DEVICE, "attention host pipeline: stream creation failed");
  }
  for (cudaEvent_t& ev : e->pipe_ev)
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      return fail(RB_E_DEVICE, "attention host pipeline: event creation failed");
    }
  e->pipe_ready = true;
  return RB_OK;
}
static std::atomic<int64_t> g_launches{0};

static int ensure_engine(Engine** out) {
  if (!g_engine) return fail(RB_E_IO, "rb_init() has not been called");
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != g_engine->device) RB_CUDA(cudaSetDevice(g_engine->device), "cudaSetDevice");
  *out = g_engine;
  return RB_OK;
}

// ------------------------------------------------------------------ internal accessors
// Used by entry points that live in other translation units (noalloc.cu).
int report_error(int rc, const char* msg) { return fail(rc, "%s", msg); }

void count_launches(int n) { g_launches += n; }

bool make_output_map(CUtensorMap* map, void* y, int y_dtype, int64_t m, int64_t n) {
  return output_map(map, y, y_dtype, m, n);
}

int w8a8_view(int64_t id, W8A8View* v) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  auto it = e->weights.find(id);
  if (it == e->weights.end() || it->second.kind != RB_WEIGHT_W8A8)
    return fail(RB_E_SHAPE, "weight id %lld is not a W8A8 weight", (long long)id);
  const Weight& w = it->second;
  v->codes = w.codes;
  v->w_scale = reinterpret_cast<const float*>(w.scales);
  v->n = w.n;
  v->k = w.k;
  v->in_scale = w.in_scale;
  v->out_scale = w.out_scale;
  v->act = w.act;
  for (int i = 0; i < 4; ++i) v->tm_codes[i] = w.tm_codes[i];
  v->err = e->err;
  v->num_sms = e->num_sms;
  v->device = e->device;
  return RB_OK;
}

static size_t dtype_bytes(int dt) {
  switch (dt) {
    case RB_DTYPE_F32: return 4;
    case RB_DTYPE_F16: return 2;
    case RB_DTYPE_BF16: return 2;
    default: return 0;
  }
}

// ------------------------------------------------------------------ ops
// pre_scale != null: x holds W8A8 activation codes int8 [m, k] with these
// per-row scales (as rb_quantize_rows_i8 / rb_add_layer_norm_quant give).
static int matmul_locked(Engine* e, int64_t id, const void* x, int x_dtype, int64_t m,
                         int64_t k, void* y, int y_dtype, cudaStream_t st, const float* pre_scale = nullptr) {
  auto it = e->weights.find(id);
  if (it == e->weights.end()) return fail(RB_E_SHAPE, "weight id %lld is not packed", (long long)id);
  const Weight& w = it->second;
  if (k != w.k) return fail(RB_E_SHAPE, "activation K=%lld mismatch for weight id %lld (K=%lld)",
                            (long long)k, (long long)id, (long long)w.k);
  if (m <= 0) return fail(RB_E_SHAPE, "matmul needs M > 0 (M=%lld)", (long long)m);
  if (m > (int64_t(1) << 31) - 1) return fail(RB_E_SHAPE, "M=%lld too large", (long long)m);
  if (!dtype_bytes(x_dtype) || !dtype_bytes(y_dtype)) return fail(RB_E_SHAPE, "bad dtype");
  const int64_t n_out = w.gated ? w.n / 2 : w.n;
  if ((n_out * static_cast<int64_t>(dtype_bytes(y_dtype))) % 16 != 0 &&
      (reinterpret_cast<uintptr_t>(y) & 15) != 0)
    return fail(RB_E_SHAPE, "output buffer must be 16-byte aligned");
  if (w.gated && (y_dtype != RB_DTYPE_F16 || (reinterpret_cast<uintptr_t>(y) & 15) != 0))
    return fail(RB_E_SHAPE, "gated (SwiGLU) weight: the output must be a 16-byte aligned f16 buffer");
  if (w.act != RB_ACT_NONE && y_dtype != RB_DTYPE_F16)
    return fail(RB_E_SHAPE, "weight id %lld has a fused activation: the output must be f16", (long long)id);

  GemmLaunch L{};
  L.M = static_cast<int>(m);
  L.N = static_cast<int>(w.n);
  L.K = static_cast<int>(w.k);
  L.out = y;
  L.ldo = static_cast<int>(n_out);
  L.gated = w.gated ? 1 : 0;
  L.act = w.act;
  L.out_dtype = y_dtype;
  L.err = e->err;
  L.num_sms = e->num_sms;
  int rc;
  if (w.kind == RB_WEIGHT_F16) {
    // fp16-resident weight (the reference's default pack, ext.rs:829-934):
    // f16 x f16 with f32 accumulation.
    const void* a = x;
    if (x_dtype != RB_DTYPE_F16 || (reinterpret_cast<uintptr_t>(x) & 15) != 0) {
      if ((rc = e->act.grow(static_cast<size_t>(m) * k * 2, "matmul activations")) != RB_OK) return rc;
      if ((rc = launch_cast(x, x_dtype, e->act.ptr, RB_DTYPE_F16, m * k, st)) != RB_OK)
        return fail(rc, "activation cast launch failed");
      g_launches++;
      a = e->act.ptr;
      L.pdl = 1;  // the GEMM's prologue (and Q8_0 weight staging) overlaps the cast
    }
    const GemmPlan plan = gemm_plan(true, L.M, L.N, L.K, e->num_sms);
    CUtensorMap tmA, tmC;
    if ((rc = make_tmap_2d(&tmA, a, 2, m, k, k, 64, plan.a_rows(), 128)) != RB_OK) return rc;
    const bool tstore = output_map(&tmC, y, y_dtype, m, w.n);
    if ((rc = launch_f16_gemm(L, plan, tmA, w.tm_codes[bn_index(plan.weight_rows())], tstore ? &tmC : nullptr,
                              st)) != RB_OK)
      return fail(rc, "f16 gemm launch failed");
    g_launches++;
    return RB_OK;
  }
  if (w.kind == RB_WEIGHT_Q8_0) {
    const void* a = x;
    if (x_dtype != RB_DTYPE_F16 || (reinterpret_cast<uintptr_t>(x) & 15) != 0) {
      if ((rc = e->act.grow(static_cast<size_t>(m) * k * 2, "matmul activations")) != RB_OK) return rc;
      if ((rc = launch_cast(x, x_dtype, e->act.ptr, RB_DTYPE_F16, m * k, st)) != RB_OK)
        return fail(rc, "activation cast launch failed");
      g_launches++;
      a = e->act.ptr;
      L.pdl = 1;  // the GEMM's prologue (and Q8_0 weight staging) overlaps the cast
    }
    // 96-column CTA-pair tiles only where the epilogue stores whole 32-column
    // f32 chunks (2-byte outputs take 64-column chunks).
    GemmPlan plan = gemm_plan(false, L.M, L.N, L.K, e->num_sms, y_dtype == RB_DTYPE_F32 && !w.gated);
    // The gated epilogue turns 128 accumulator columns into 64 outputs: tiles
    // of 256 or 128 columns.
    if (w.gated && plan.bn % 128 != 0) plan = GemmPlan{plan.pair ? 256 : 128, 1, plan.pair};
    CUtensorMap tmA, tmC;
    if ((rc = make_tmap_2d(&tmA, a, 2, m, k, k, 64, plan.a_rows(), 128)) != RB_OK) return rc;
    const bool tstore = output_map(&tmC, y, y_dtype, m, n_out);
    if (w.gated && !tstore) return fail(RB_E_SHAPE, "gated weight: output tensor map unavailable");
    // The pair kernel reads Q8_0 codes and scales from global memory, not
    // through these maps (a 96-column pair tile has no map of its own).
    const int bi = bn_index(plan.weight_rows()) < 0 ? 0 : bn_index(plan.weight_rows());
    L.w_codes = w.codes;
    L.w_scales = w.scales;
    L.w_pitch = w.pitch;
    L.w_rows = w.n;
    if ((rc = launch_q8_gemm(L, plan, tmA, w.tm_codes[bi], w.tm_scales[bi], tstore ? &tmC : nullptr,
                             st)) != RB_OK)
      return fail(rc, "q8_0 gemm launch failed");
    g_launches++;
    return RB_OK;
  }
  if (w.kind == RB_WEIGHT_I8G) {
    // Group-wise int8: the activation group quantiser, then one GEMM whose
    // fold warps promote each group's exact int32 partial into the f32 result
    // in group order (no partial leaves the SM).
    const int64_t G = w.group, ng = k / G;
    const size_t codes_bytes = (static_cast<size_t>(m) * k + 255) & ~size_t(255);
    if ((rc = e->act.grow(codes_bytes, "int8 group activation codes")) != RB_OK) return rc;
    if ((rc = e->rowscale.grow(static_cast<size_t>(m) * ng * 4, "int8 group scales")) != RB_OK) return rc;
    int8_t* codes = reinterpret_cast<int8_t*>(e->act.ptr);
    float* a_s = reinterpret_cast<float*>(e->rowscale.ptr);
    if ((rc = launch_quantize_groups(x, x_dtype, m, k, static_cast<int>(G), codes, a_s, st)) != RB_OK)
      return fail(rc, "group quantiser launch failed");
    g_launches++;
    CUtensorMap tmA, tmB, tmC;
    if ((rc = make_tmap_2d(&tmA, codes, 1, m, k, k, 128, 128, 128)) != RB_OK) return rc;
    if ((rc = make_tmap_2d(&tmB, w.codes, 1, w.n, k, k, 128, 128, 128)) != RB_OK) return rc;
    const bool tstore = output_map(&tmC, y, y_dtype, m, w.n);
    if ((rc = launch_i8g_gemm(static_cast<int>(m), static_cast<int>(w.n), static_cast<int>(k), static_cast<int>(G),
                              a_s, w.scales_t, static_cast<int>(w.ldb), y, y_dtype, tmA, tmB,
                              tstore ? &tmC : nullptr, e->err, e->num_sms, st)) != RB_OK)
      return fail(rc, "int8 group gemm launch failed");
    g_launches++;
    return RB_OK;
  }
  if (w.kind == RB_WEIGHT_W8A8) {
    const int8_t* codes = reinterpret_cast<const int8_t*>(x);
    const float* rs = pre_scale;
    if (!pre_scale) {
      const size_t codes_bytes = (static_cast<size_t>(m) * k + 255) & ~size_t(255);
      if ((rc = e->act.grow(codes_bytes, "w8a8 activation codes")) != RB_OK) return rc;
      if ((rc = e->rowscale.grow(static_cast<size_t>(m) * 4, "w8a8 row scales")) != RB_OK) return rc;
      int8_t* c8 = reinterpret_cast<int8_t*>(e->act.ptr);
      float* r32 = reinterpret_cast<float*>(e->rowscale.ptr);
      if ((rc = launch_quantize_rows_i8(x, x_dtype, m, k, w.in_scale, c8, r32, st)) != RB_OK)
        return fail(rc, "row quantiser launch failed");
      g_launches++;
      codes = c8;
      rs = r32;
      L.pdl = 1;  // the GEMM's prologue overlaps the quantiser
    } else if ((reinterpret_cast<uintptr_t>(x) & 15) != 0 || k % 16 != 0) {
      return fail(RB_E_SHAPE, "w8a8 codes input: 16-byte aligned rows needed (k %% 16 == 0)");
    }
    CUtensorMap tmA, tmC;
    if ((rc = make_tmap_2d(&tmA, codes, 1, m, k, k, 128, 128, 128)) != RB_OK) return rc;
    L.s_row = rs;
    L.s_col = reinterpret_cast<const float*>(w.scales);
    L.out_scale = w.out_scale;
    const bool tstore = output_map(&tmC, y, y_dtype, m, w.n);
    const GemmPlan plan = gemm_plan(true, L.M, L.N, L.K, e->num_sms);
    if ((rc = launch_w8a8_gemm(L, plan, tmA, w.tm_codes[bn_index(plan.weight_rows())], tstore ? &tmC : nullptr,
                               st)) != RB_OK)
      return fail(rc, "w8a8 gemm launch failed");
    g_launches++;
    return RB_OK;
  }
  return fail(RB_E_UNSUPPORTED, "weight kind %d", w.kind);
}

static int attention_locked(Engine* e, const void* q, int64_t ldq, const void* k, int64_t ldk,
                            const void* v, int64_t ldv, void* out, int64_t ldo, int dtype,
                            int64_t batch, int64_t n_q, int64_t n_kv, int n_head, int n_kv_heads,
                            int head_dim, float scale, float softcap, int mask_mode, int64_t window,
                            int64_t q_start, int64_t kv_start, cudaStream_t st) {
  // Contract of check_flash (attn/mod.rs:1424-1460) and attention_impl
  // (ext.rs:1680-1712).
  if (n_q <= 0 || n_kv <= 0 || head_dim <= 0 || batch <= 0)
    return fail(RB_E_SHAPE, "flash_attn/dims: n_q=%lld n_kv=%lld head_dim=%d batch=%lld",
                (long long)n_q, (long long)n_kv, head_dim, (long long)batch);
  if (n_head <= 0 || n_kv_heads <= 0 || n_head % n_kv_heads != 0)
    return fail(RB_E_SHAPE, "flash_attn/heads: n_head=%d n_kv_heads=%d", n_head, n_kv_heads);
  if (head_dim != 64 && head_dim != 128 && head_dim != 72)
    return fail(RB_E_UNSUPPORTED, "flash_attn/dims: head_dim %d (supported: 64, 72, 128)", head_dim);
  if (mask_mode < RB_MASK_NONE || mask_mode > RB_MASK_CAUSAL_BLOCK)
    return fail(RB_E_SHAPE, "unknown mask mode %d", mask_mode);
  const bool block = mask_mode == RB_MASK_NONE_BLOCK || mask_mode == RB_MASK_WINDOW_BLOCK ||
                     mask_mode == RB_MASK_CAUSAL_BLOCK;
  if (!block && n_q != n_kv)
    return fail(RB_E_SHAPE, "the full-sequence mask modes need equal query/key lengths (%lld vs %lld)",
                (long long)n_q, (long long)n_kv);
  if (batch * n_q > (1 << 30) || batch * n_kv > (1 << 30)) return fail(RB_E_SHAPE, "sequence too long");
  if (ldq < (int64_t)n_head * head_dim || ldo < (int64_t)n_head * head_dim ||
      ldk < (int64_t)n_kv_heads * head_dim || ldv < (int64_t)n_kv_heads * head_dim)
    return fail(RB_E_SHAPE, "flash_attn/buffers: row strides shorter than heads * head_dim");
  // Windowed modes with window < 0 fall back to their unwindowed form
  // (ext.rs:672-677, 693-698, 717-727).
  if (mask_mode == RB_MASK_WINDOW && window < 0) mask_mode = RB_MASK_NONE;
  if (mask_mode == RB_MASK_CAUSAL_WINDOW && window < 0) mask_mode = RB_MASK_CAUSAL;
  if (mask_mode == RB_MASK_WINDOW_BLOCK && window < 0) mask_mode = RB_MASK_NONE_BLOCK;
  if (q_start < 0) q_start = 0;
  if (kv_start < 0) kv_start = 0;

  int rc;
  const void* qh = q;
  const void* kh = k;
  const void* vh = v;
  void* oh = out;
  int kdt = dtype;
  const int64_t wq = (int64_t)n_head * head_dim, wk = (int64_t)n_kv_heads * head_dim;
  if (dtype == RB_DTYPE_F32) {
    // f32 tensors (the Burn boundary) are rounded to f16 like fill_heads
    // (ext.rs:2174-2190), and the f16 result widened on the way out.
    if (ldq != wq || ldk != wk || ldv != wk || ldo != wq)
      return fail(RB_E_UNSUPPORTED, "f32 attention needs contiguous [S, heads*d] tensors");
    const size_t nq = static_cast<size_t>(batch * n_q) * wq;
    const size_t nk = static_cast<size_t>(batch * n_kv) * wk;
    const size_t a16 = (nq * 2 + 255) & ~size_t(255), k16 = (nk * 2 + 255) & ~size_t(255);
    if ((rc = e->act.grow(2 * a16 + 2 * k16, "attention f16 staging")) != RB_OK) return rc;
    uint8_t* base = reinterpret_cast<uint8_t*>(e->act.ptr);
    void* q16 = base;
    void* o16 = base + a16;
    void* k16p = base + 2 * a16;
    void* v16 = base + 2 * a16 + k16;
    if ((rc = launch_cast(q, RB_DTYPE_F32, q16, RB_DTYPE_F16, nq, st)) != RB_OK) return fail(rc, "cast q");
    if ((rc = launch_cast(k, RB_DTYPE_F32, k16p, RB_DTYPE_F16, nk, st)) != RB_OK) return fail(rc, "cast k");
    if ((rc = launch_cast(v, RB_DTYPE_F32, v16, RB_DTYPE_F16, nk, st)) != RB_OK) return fail(rc, "cast v");
    g_launches += 3;
    qh = q16; kh = k16p; vh = v16; oh = o16;
    kdt = RB_DTYPE_F16;
  } else if (dtype != RB_DTYPE_F16 && dtype != RB_DTYPE_BF16) {
    return fail(RB_E_SHAPE, "attention dtype %d", dtype);
  }
  // head_dim 72 is staged as 80 (the UMMA K granularity) straight from the
  // caller's rows: [rows, heads, 72] maps whose 16-column tail atom covers
  // head columns 64..79, the last 8 past the head and so zero-filled by TMA.
  // The output keeps 72 columns.
  const int d_stage = head_dim == 72 ? 80 : head_dim;
  const int64_t sq = ldq, sk = ldk, sv = ldv, cq = wq, ck = wk;
  CUtensorMap tm[6];
  // Q tiles are 128 query rows, K/V tiles kAttnKeyTile keys; 64-element
  // (128-B) column atoms, plus 16-element (32-B) tail atoms for the 72-wide heads.
  constexpr uint32_t kt = kAttnKeyTile;
  if (head_dim == 72) {
    const uint64_t rq = batch * n_q, rk = batch * n_kv;
    if ((rc = make_tmap_heads(&tm[0], qh, rq, n_head, 72, sq, 64, 128, 128)) != RB_OK ||
        (rc = make_tmap_heads(&tm[1], kh, rk, n_kv_heads, 72, sk, 64, kt, 128)) != RB_OK ||
        (rc = make_tmap_heads(&tm[2], vh, rk, n_kv_heads, 72, sv, 64, kt, 128)) != RB_OK ||
        (rc = make_tmap_heads(&tm[3], qh, rq, n_head, 72, sq, 16, 128, 32)) != RB_OK ||
        (rc = make_tmap_heads(&tm[4], kh, rk, n_kv_heads, 72, sk, 16, kt, 32)) != RB_OK ||
        (rc = make_tmap_heads(&tm[5], vh, rk, n_kv_heads, 72, sv, 16, kt, 32)) != RB_OK)
      return rc;
  } else {
    if ((rc = make_tmap_2d(&tm[0], qh, 2, batch * n_q, cq, sq, 64, 128, 128)) != RB_OK) return rc;
    if ((rc = make_tmap_2d(&tm[1], kh, 2, batch * n_kv, ck, sk, 64, kt, 128)) != RB_OK) return rc;
    if ((rc = make_tmap_2d(&tm[2], vh, 2, batch * n_kv, ck, sv, 64, kt, 128)) != RB_OK) return rc;
    tm[3] = tm[0];
    tm[4] = tm[1];
    tm[5] = tm[2];
  }
  if ((reinterpret_cast<uintptr_t>(oh) & 15) != 0 || (ldo * 2) % 16 != 0)
    return fail(RB_E_SHAPE, "attention output must be 16-byte aligned");
  AttnLaunch L{};
  L.q = qh; L.k = kh; L.v = vh; L.out = oh;
  L.dtype = kdt;
  L.batch = static_cast<int>(batch);
  L.n_q = static_cast<int>(n_q);
  L.n_kv = static_cast<int>(n_kv);
  L.n_head = n_head;
  L.n_kv_heads = n_kv_heads;
  L.head_dim = d_stage;
  L.head_maps = head_dim == 72 ? 1 : 0;
  L.d_out = head_dim;
  L.ldq = static_cast<int>(sq);
  L.ldk = static_cast<int>(sk);
  L.ldv = static_cast<int>(sv);
  L.ldo = static_cast<int>(ldo);
  L.scale = scale;
  L.softcap = softcap;
  L.mask_mode = mask_mode;
  L.window = window;
  L.q_start = q_start;
  L.kv_start = kv_start;
  L.err = e->err;
  L.num_sms = e->num_sms;
  L.ws_rec = e->attn_rec;
  L.ws_cnt = e->attn_cnt;
  g_last_error.clear();
  if ((rc = launch_attention(tm, L, st)) != RB_OK) {
    const std::string why = g_last_error;
    return fail(rc, "attention launch failed%s%s", why.empty() ? "" : ": ", why.c_str());
  }
  g_launches++;
  if (dtype == RB_DTYPE_F32) {
    if ((rc = launch_cast(oh, RB_DTYPE_F16, out, RB_DTYPE_F32, batch * n_q * wq, st)) != RB_OK)
      return fail(rc, "cast out");
    g_launches++;
  }
  return RB_OK;
}

}  // namespace rb

using namespace rb;

extern "C" {

int rb_init(int device_ordinal) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_engine) return RB_OK;
  int count = 0;
  RB_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (device_ordinal < 0 || device_ordinal >= count)
    return fail(RB_E_DEVICE, "device %d out of range (%d devices)", device_ordinal, count);
  RB_CUDA(cudaSetDevice(device_ordinal), "cudaSetDevice");
  cudaDeviceProp prop;
  RB_CUDA(cudaGetDeviceProperties(&prop, device_ordinal), "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(RB_E_UNSUPPORTED, "device %d is sm_%d%d; librocket_b200 needs sm_100a", device_ordinal,
                prop.major, prop.minor);
  if (!load_encode_fn()) return fail(RB_E_DEVICE, "cuTensorMapEncodeTiled unavailable");
  Engine* e = new Engine();
  e->device = device_ordinal;
  e->num_sms = prop.multiProcessorCount;
  if (cudaMalloc(&e->err, sizeof(uint32_t)) != cudaSuccess) {
    delete e;
    return fail(RB_E_NOMEM, "cudaMalloc(error word) failed");
  }
  cudaMemset(e->err, 0, sizeof(uint32_t));
  // Attention split-mode workspace; without it attention runs one CTA per unit.
  if (cudaMalloc(&e->attn_rec, kAttnRecBytes) != cudaSuccess ||
      cudaMalloc(&e->attn_cnt, kAttnCntBytes) != cudaSuccess ||
      cudaMemset(e->attn_cnt, 0, kAttnCntBytes) != cudaSuccess) {
    cudaGetLastError();
    if (e->attn_rec) cudaFree(e->attn_rec);
    if (e->attn_cnt) cudaFree(e->attn_cnt);
    e->attn_rec = nullptr;
    e->attn_cnt = nullptr;
  }
  cudaStreamCreateWithFlags(&e->host_stream, cudaStreamNonBlocking);
  g_engine = e;
  return RB_OK;
}

int rb_last_error(char* buf, size_t len) {
  if (buf && len) {
    std::strncpy(buf, g_last_error.c_str(), len - 1);
    buf[len - 1] = '\0';
  }
  return static_cast<int>(g_last_error.size());
}

int rb_check_device_errors(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  RB_CUDA(cudaDeviceSynchronize(), "device synchronize");
  uint32_t word = 0;
  RB_CUDA(cudaMemcpy(&word, e->err, sizeof(word), cudaMemcpyDeviceToHost), "read error word");
  if (word) {
    cudaMemset(e->err, 0, sizeof(uint32_t));
    // An aborted attention launch can leave split-mode counters mid-count.
    if (e->attn_cnt) cudaMemset(e->attn_cnt, 0, kAttnCntBytes);
    return fail(RB_E_DEVICE, "kernel error word 0x%x (%s%s%s%s)", word,
                (word & kErrWaitTimeout) ? "wait-timeout " : "",
                (word & kErrTmemAlloc) ? "tmem-alloc " : "",
                (word & kErrBadShape) ? "bad-shape " : "",
                (word & kErrOverflow) ? "exchange-capacity-overflow" : "");
  }
  return RB_OK;
}

int64_t rb_pack_q8_0(const void* blocks_host, int64_t n, int64_t k) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!blocks_host) return fail(RB_E_SHAPE, "null Q8_0 blocks");
  if (n <= 0 || k <= 0 || k % 32 != 0)
    return fail(RB_E_SHAPE, "Q8_0 weight [%lld, %lld]: K must be a positive multiple of 32",
                (long long)n, (long long)k);
  if (n > (1 << 30) || k > (1 << 30)) return fail(RB_E_SHAPE, "Q8_0 weight too large");
  const size_t nblk = static_cast<size_t>(n) * (k / 32);
  Weight w;
  w.kind = RB_WEIGHT_Q8_0;
  w.n = n;
  w.k = k;
  w.pitch = (n + 7) & ~int64_t(7);
  const size_t sbytes = static_cast<size_t>(w.pitch) * (k / 32) * 2;
  uint8_t* dblk = nullptr;
  if (cudaMalloc(&dblk, nblk * 34) != cudaSuccess ||
      cudaMalloc(&w.codes, static_cast<size_t>(n) * k) != cudaSuccess ||
      cudaMalloc(&w.scales, sbytes) != cudaSuccess) {
    cudaGetLastError();
    if (dblk) cudaFree(dblk);
    if (w.codes) cudaFree(w.codes);
    return fail(RB_E_NOMEM, "Q8_0 pack: device allocation failed");
  }
  RB_CUDA(cudaMemcpy(dblk, blocks_host, nblk * 34, cudaMemcpyHostToDevice), "Q8_0 upload");
  cudaMemset(w.scales, 0, sbytes);
  if ((rc = launch_q8_0_unpack_blocks(dblk, n, k, w.pitch, w.codes, reinterpret_cast<uint16_t*>(w.scales),
                                      nullptr)) != RB_OK)
    return fail(rc, "Q8_0 unpack launch failed");
  g_launches++;
  RB_CUDA(cudaDeviceSynchronize(), "Q8_0 unpack");
  cudaFree(dblk);
  w.bytes = static_cast<size_t>(n) * k + sbytes;
  if ((rc = weight_maps(w)) != RB_OK) return rc;
  const int64_t id = e->next_id++;
  e->weights[id] = w;
  return id;
}

static int64_t pack_f32_q8_0_impl(const float* const* parts_host, const int64_t* n_parts, int num_parts,
                                  int64_t k, cudaMemcpyKind kind) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (num_parts < 1 || !parts_host || !n_parts) return fail(RB_E_SHAPE, "no weight parts");
  if (k <= 0 || k % 32 != 0) return fail(RB_E_SHAPE, "Q8_0 pack: K=%lld must be a positive multiple of 32", (long long)k);
  int64_t n = 0;
  for (int i = 0; i < num_parts; ++i) {
    if (n_parts[i] <= 0 || !parts_host[i]) return fail(RB_E_SHAPE, "weight part %d is empty", i);
    n += n_parts[i];
  }
  if (n > (1 << 30)) return fail(RB_E_SHAPE, "Q8_0 weight too large");
  Weight w;
  w.kind = RB_WEIGHT_Q8_0;
  w.n = n;
  w.k = k;
  w.pitch = (n + 7) & ~int64_t(7);
  const size_t sbytes = static_cast<size_t>(w.pitch) * (k / 32) * 2;
  float* dw = nullptr;
  if (cudaMalloc(&dw, static_cast<size_t>(n) * k * 4) != cudaSuccess ||
      cudaMalloc(&w.codes, static_cast<size_t>(n) * k) != cudaSuccess ||
      cudaMalloc(&w.scales, sbytes) != cudaSuccess) {
    cudaGetLastError();
    if (dw) cudaFree(dw);
    if (w.codes) cudaFree(w.codes);
    return fail(RB_E_NOMEM, "Q8_0 pack: device allocation failed");
  }
  int64_t off = 0;
  for (int i = 0; i < num_parts; ++i) {
    RB_CUDA(cudaMemcpy(dw + off * k, parts_host[i], static_cast<size_t>(n_parts[i]) * k * 4, kind),
            "weight upload");
    off += n_parts[i];
  }
  cudaMemset(w.scales, 0, sbytes);
  if ((rc = launch_q8_0_encode(dw, n, k, w.pitch, w.codes, reinterpret_cast<uint16_t*>(w.scales), nullptr)) != RB_OK)
    return fail(rc, "Q8_0 encode launch failed");
  g_launches++;
  RB_CUDA(cudaDeviceSynchronize(), "Q8_0 encode");
  cudaFree(dw);
  w.bytes = static_cast<size_t>(n) * k + sbytes;
  if ((rc = weight_maps(w)) != RB_OK) return rc;
  const int64_t id = e->next_id++;
  e->weights[id] = w;
  return id;
}

int64_t rb_pack_f32_q8_0(const float* const* parts_host, const int64_t* n_parts, int num_parts,
                         int64_t k) {
  return pack_f32_q8_0_impl(parts_host, n_parts, num_parts, k, cudaMemcpyHostToDevice);
}

int64_t rb_pack_f32_q8_0_device(const float* const* parts_dev, const int64_t* n_parts, int num_parts,
                                int64_t k) {
  return pack_f32_q8_0_impl(parts_dev, n_parts, num_parts, k, cudaMemcpyDeviceToDevice);
}

int64_t rb_pack_f32_q8_0_gated_device(const float* gate_dev, const float* up_dev, int64_t n_inter, int64_t k) {
  if (!gate_dev || !up_dev || n_inter <= 0 || n_inter % 64 != 0 || k <= 0)
    return fail(RB_E_SHAPE, "gated pack: gate/up [%lld, %lld] need rows a positive multiple of 64",
                (long long)n_inter, (long long)k);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    Engine* e;
    int rc = ensure_engine(&e);
    if (rc) return rc;
  }
  // Interleave 32-row blocks: rows [64b, 64b+32) = gate block b, [64b+32, 64b+64) = up block b.
  float* inter = nullptr;
  const size_t blk = static_cast<size_t>(32) * k * sizeof(float);
  if (cudaMalloc(&inter, 2 * static_cast<size_t>(n_inter) * k * sizeof(float)) != cudaSuccess) {
    cudaGetLastError();
    return fail(RB_E_NOMEM, "gated pack: staging allocation failed");
  }
  const size_t nb = static_cast<size_t>(n_inter / 32);
  if (cudaMemcpy2D(inter, 2 * blk, gate_dev, blk, blk, nb, cudaMemcpyDeviceToDevice) != cudaSuccess ||
      cudaMemcpy2D(reinterpret_cast<uint8_t*>(inter) + blk, 2 * blk, up_dev, blk, blk, nb,
                   cudaMemcpyDeviceToDevice) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(inter);
    return fail(RB_E_DEVICE, "gated pack: interleave copy failed");
  }
  const float* parts[1] = {inter};
  const int64_t ns[1] = {2 * n_inter};
  const int64_t id = pack_f32_q8_0_impl(parts, ns, 1, k, cudaMemcpyDeviceToDevice);
  cudaDeviceSynchronize();
  cudaFree(inter);
  if (id > 0) {
    std::lock_guard<std::mutex> lk(g_mu);
    g_engine->weights[id].gated = true;
  }
  return id;
}

int64_t rb_pack_w8a8(const int8_t* codes_host, const float* w_scale_host, int64_t n, int64_t k,
                     float in_scale, float out_scale) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  // pack_qat asserts (ext.rs:1390-1394); this build tiles any K % 16 == 0
  // (TMA row pitch) and any N.
  if (!codes_host || !w_scale_host) return fail(RB_E_SHAPE, "null W8A8 codes/scales");
  if (n <= 0 || k <= 0 || k % 16 != 0)
    return fail(RB_E_SHAPE, "W8A8 weight [%lld, %lld]: K must be a positive multiple of 16",
                (long long)n, (long long)k);
  if (!(in_scale >= 0.0f)) return fail(RB_E_SHAPE, "QAT input scale must not be negative");
  if (n > (1 << 30) || k > (1 << 30)) return fail(RB_E_SHAPE, "W8A8 weight too large");
  Weight w;
  w.kind = RB_WEIGHT_W8A8;
  w.n = n;
  w.k = k;
  w.in_scale = in_scale;
  w.out_scale = out_scale;
  if (cudaMalloc(&w.codes, static_cast<size_t>(n) * k) != cudaSuccess ||
      cudaMalloc(&w.scales, static_cast<size_t>(n) * 4) != cudaSuccess) {
    cudaGetLastError();
    if (w.codes) cudaFree(w.codes);
    return fail(RB_E_NOMEM, "W8A8 pack: device allocation failed");
  }
  RB_CUDA(cudaMemcpy(w.codes, codes_host, static_cast<size_t>(n) * k, cudaMemcpyHostToDevice), "codes upload");
  RB_CUDA(cudaMemcpy(w.scales, w_scale_host, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice), "scale upload");
  if ((rc = weight_maps(w)) != RB_OK) return rc;
  w.bytes = static_cast<size_t>(n) * k + static_cast<size_t>(n) * 4;
  const int64_t id = e->next_id++;
  e->weights[id] = w;
  return id;
}

int64_t rb_pack_f16(const void* const* parts_host, const int64_t* n_parts, int num_parts, int64_t k,
                    int src_dtype) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!parts_host || !n_parts || num_parts <= 0) return fail(RB_E_SHAPE, "pack: no parts");
  if (k <= 0 || k % 8 != 0) return fail(RB_E_SHAPE, "pack: K=%lld must be a positive multiple of 8", (long long)k);
  const int eb = dtype_bytes(src_dtype);
  if (!eb) return fail(RB_E_SHAPE, "pack: bad source dtype %d", src_dtype);
  int64_t n = 0;
  for (int i = 0; i < num_parts; ++i) {
    if (!parts_host[i] || n_parts[i] <= 0) return fail(RB_E_SHAPE, "pack: empty part %d", i);
    n += n_parts[i];
  }
  if (n > (1 << 30) || k > (1 << 30)) return fail(RB_E_SHAPE, "pack: weight too large");
  Weight w;
  w.kind = RB_WEIGHT_F16;
  w.n = n;
  w.k = k;
  void* tmp = nullptr;
  const size_t elems = static_cast<size_t>(n) * k;
  if (cudaMalloc(&w.codes, elems * 2) != cudaSuccess ||
      (src_dtype != RB_DTYPE_F16 && cudaMalloc(&tmp, elems * eb) != cudaSuccess)) {
    cudaGetLastError();
    if (w.codes) cudaFree(w.codes);
    return fail(RB_E_NOMEM, "pack: device allocation failed");
  }
  // parts concatenated along N (pack2 / pack3 / pack_seg, ext.rs:852-934)
  uint8_t* dst = src_dtype == RB_DTYPE_F16 ? reinterpret_cast<uint8_t*>(w.codes) : reinterpret_cast<uint8_t*>(tmp);
  size_t off = 0;
  for (int i = 0; i < num_parts; ++i) {
    const size_t bytes = static_cast<size_t>(n_parts[i]) * k * eb;
    RB_CUDA(cudaMemcpy(dst + off, parts_host[i], bytes, cudaMemcpyHostToDevice), "weight upload");
    off += bytes;
  }
  if (src_dtype != RB_DTYPE_F16) {
    // f32 / bf16 -> f16 RNE, as the reference's pack converts (f32_to_f16_par, ext.rs:2144-2156)
    rc = launch_cast(tmp, src_dtype, w.codes, RB_DTYPE_F16, static_cast<int64_t>(elems), nullptr);
    g_launches++;
    const cudaError_t ce = cudaDeviceSynchronize();
    cudaFree(tmp);
    if (rc != RB_OK || ce != cudaSuccess) return fail(RB_E_DEVICE, "pack: f16 conversion failed");
  }
  if ((rc = weight_maps(w)) != RB_OK) return rc;
  w.bytes = elems * 2;
  const int64_t id = e->next_id++;
  e->weights[id] = w;
  return id;
}

int64_t rb_pack_i8(const float* w_host, int64_t n, int64_t k, int64_t group) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!w_host) return fail(RB_E_SHAPE, "null weight");
  // pack_i8_one asserts (ext.rs:948-953): group a positive multiple of 32
  // dividing K; this build takes any N.
  if (n <= 0 || k <= 0 || group <= 0 || group % 32 || k % group)
    return fail(RB_E_SHAPE, "int8 group %lld must be a positive multiple of 32 dividing K=%lld", (long long)group,
                (long long)k);
  if (n > (1 << 30) || k > (1 << 30)) return fail(RB_E_SHAPE, "int8 weight too large");
  Weight w;
  w.kind = RB_WEIGHT_I8G;
  w.n = n;
  w.k = k;
  w.group = group;
  const size_t ng = static_cast<size_t>(k / group);
  float* tmp = nullptr;
  if (cudaMalloc(&w.codes, static_cast<size_t>(n) * k) != cudaSuccess ||
      cudaMalloc(&w.scales, static_cast<size_t>(n) * ng * 4) != cudaSuccess ||
      cudaMalloc(&tmp, static_cast<size_t>(n) * k * 4) != cudaSuccess) {
    cudaGetLastError();
    if (w.codes) cudaFree(w.codes);
    if (w.scales) cudaFree(w.scales);
    return fail(RB_E_NOMEM, "int8 pack: device allocation failed");
  }
  RB_CUDA(cudaMemcpy(tmp, w_host, static_cast<size_t>(n) * k * 4, cudaMemcpyHostToDevice), "weight upload");
  rc = launch_quantize_groups(tmp, RB_DTYPE_F32, n, k, static_cast<int>(group), w.codes,
                              reinterpret_cast<float*>(w.scales), nullptr);
  g_launches++;
  const cudaError_t ce = cudaDeviceSynchronize();
  cudaFree(tmp);
  if (rc != RB_OK || ce != cudaSuccess) return fail(RB_E_DEVICE, "int8 group quantiser failed");
  // Group-major copy of the scales for the GEMM's fold warps (one 16-byte
  // load gives four columns' scales of a group), zero-padded to whole tiles.
  w.ldb = (n + 127) / 128 * 128;
  {
    std::vector<float> s(static_cast<size_t>(n) * ng), st(static_cast<size_t>(w.ldb) * ng, 0.0f);
    RB_CUDA(cudaMemcpy(s.data(), w.scales, s.size() * 4, cudaMemcpyDeviceToHost), "int8 scales download");
    for (int64_t r = 0; r < n; ++r)
      for (size_t g = 0; g < ng; ++g) st[g * w.ldb + r] = s[r * ng + g];
    if (cudaMalloc(&w.scales_t, st.size() * 4) != cudaSuccess) {
      cudaGetLastError();
      cudaFree(w.codes);
      cudaFree(w.scales);
      return fail(RB_E_NOMEM, "int8 pack: device allocation failed");
    }
    RB_CUDA(cudaMemcpy(w.scales_t, st.data(), st.size() * 4, cudaMemcpyHostToDevice), "int8 scales upload");
  }
  w.bytes = static_cast<size_t>(n) * k + static_cast<size_t>(n) * ng * 4 + static_cast<size_t>(w.ldb) * ng * 4;
  const int64_t id = e->next_id++;
  e->weights[id] = w;
  return id;
}

int rb_quantize_row_groups(const void* x, int x_dtype, int64_t m, int64_t k, int64_t group, int8_t* codes,
                           float* scales, void* stream) {
  if (!x || !codes || !scales || m <= 0 || k <= 0 || group <= 0 || k % group)
    return fail(RB_E_SHAPE, "quantize_row_groups: group must divide K");
  const int rc = launch_quantize_groups(x, x_dtype, m, k, static_cast<int>(group), codes, scales,
                                        reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "quantize_row_groups: bad dtype");
}

int64_t rb_pack_f32_w8a8_device(const float* w_dev, int64_t n, int64_t k, float in_scale,
                                float out_scale) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!w_dev) return fail(RB_E_SHAPE, "null weight");
  if (n <= 0 || k <= 0 || k % 16 != 0)
    return fail(RB_E_SHAPE, "W8A8 weight [%lld, %lld]: K must be a positive multiple of 16",
                (long long)n, (long long)k);
  if (!(in_scale >= 0.0f)) return fail(RB_E_SHAPE, "QAT input scale must not be negative");
  Weight w;
  w.kind = RB_WEIGHT_W8A8;
  w.n = n;
  w.k = k;
  w.in_scale = in_scale;
  w.out_scale = out_scale;
  if (cudaMalloc(&w.codes, static_cast<size_t>(n) * k) != cudaSuccess ||
      cudaMalloc(&w.scales, static_cast<size_t>(n) * 4) != cudaSuccess) {
    cudaGetLastError();
    if (w.codes) cudaFree(w.codes);
    return fail(RB_E_NOMEM, "W8A8 pack: device allocation failed");
  }
  if ((rc = launch_w8a8_weight_quant(w_dev, n, k, w.codes, reinterpret_cast<float*>(w.scales), nullptr)) != RB_OK)
    return fail(rc, "W8A8 weight quantiser launch failed");
  g_launches++;
  RB_CUDA(cudaDeviceSynchronize(), "W8A8 weight quantiser");
  if ((rc = weight_maps(w)) != RB_OK) return rc;
  w.bytes = static_cast<size_t>(n) * k + static_cast<size_t>(n) * 4;
  const int64_t id = e->next_id++;
  e->weights[id] = w;
  return id;
}

int rb_weight_info(int64_t id, int* kind, int64_t* n, int64_t* k) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  auto it = e->weights.find(id);
  if (it == e->weights.end()) return fail(RB_E_SHAPE, "weight id %lld is not packed", (long long)id);
  if (kind) *kind = it->second.kind;
  if (n) *n = it->second.gated ? it->second.n / 2 : it->second.n;  // output columns
  if (k) *k = it->second.k;
  return RB_OK;
}

int rb_matmul(int64_t id, const void* x, int x_dtype, int64_t m, int64_t k, void* y, int y_dtype,
              void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!x || !y) return fail(RB_E_SHAPE, "null matmul buffer");
  return matmul_locked(e, id, x, x_dtype, m, k, y, y_dtype, reinterpret_cast<cudaStream_t>(stream));
}

int rb_matmul_w8a8_codes(int64_t id, const int8_t* codes, const float* row_scale, int64_t m, int64_t k, void* y,
                         int y_dtype, void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!codes || !row_scale || !y) return fail(RB_E_SHAPE, "null matmul buffer");
  auto it = e->weights.find(id);
  if (it == e->weights.end() || it->second.kind != RB_WEIGHT_W8A8)
    return fail(RB_E_SHAPE, "weight id %lld is not a W8A8 weight", (long long)id);
  return matmul_locked(e, id, codes, RB_DTYPE_F16, m, k, y, y_dtype, reinterpret_cast<cudaStream_t>(stream),
                       row_scale);
}

int rb_add_layer_norm_quant(float* x, const void* delta_f16, const float* g, const float* b, float eps,
                            int8_t* codes, float* row_scale, int64_t rows, int64_t d, void* stream) {
  if (!x || !g || !b || !codes || !row_scale || rows <= 0) return fail(RB_E_SHAPE, "add_layer_norm_quant: bad arguments");
  const int rc = launch_add_layer_norm_quant(x, delta_f16, g, b, eps, codes, row_scale, rows, static_cast<int>(d),
                                             reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "add_layer_norm_quant: unsupported width %lld", (long long)d);
}

int rb_matmul_host(int64_t id, const void* x_host, int x_dtype, int64_t m, int64_t k, void* y_host,
                   int y_dtype) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!x_host || !y_host) return fail(RB_E_SHAPE, "null matmul buffer");
  auto it = e->weights.find(id);
  if (it == e->weights.end()) return fail(RB_E_SHAPE, "weight id %lld is not packed", (long long)id);
  const int64_t n = it->second.gated ? it->second.n / 2 : it->second.n;  // output columns
  const size_t xb = static_cast<size_t>(m) * k * dtype_bytes(x_dtype);
  const size_t yb = static_cast<size_t>(m) * n * dtype_bytes(y_dtype);
  if (!xb || !yb) return fail(RB_E_SHAPE, "bad dtype or empty matmul");
  if ((rc = e->io_in.grow(xb, "matmul input staging")) != RB_OK) return rc;
  if ((rc = e->io_out.grow(yb, "matmul output staging")) != RB_OK) return rc;
  // Larger calls are pipelined in row chunks (whole 256-row tiles): chunk
  // c's rows go over, its matmul runs once they are on the device, and its
  // output comes back while later chunks still copy in or compute. Every
  // output row depends on its own input row only.
  if (m >= 512 && it->second.kind != RB_WEIGHT_I8G) {
    if ((rc = ensure_pipe(e)) != RB_OK) return rc;
    const int64_t rows = ((m + kHostAttnChunks - 1) / kHostAttnChunks + 255) / 256 * 256;
    cudaStream_t s_in = e->pipe_in, s_cmp = e->host_stream, s_out = e->pipe_out;
    cudaEvent_t* ev = e->pipe_ev;  // [1 + c]: chunk c in; [1 + C + c]: chunk c done
    const size_t xrow = static_cast<size_t>(k) * dtype_bytes(x_dtype), yrow = static_cast<size_t>(n) * dtype_bytes(y_dtype);
    int c = 0;
    for (int64_t r0 = 0; r0 < m; r0 += rows, ++c) {
      const int64_t nr = m - r0 < rows ? m - r0 : rows;
      uint8_t* xd = reinterpret_cast<uint8_t*>(e->io_in.ptr) + r0 * xrow;
      uint8_t* yd = reinterpret_cast<uint8_t*>(e->io_out.ptr) + r0 * yrow;
      RB_CUDA(cudaMemcpyAsync(xd, reinterpret_cast<const uint8_t*>(x_host) + r0 * xrow, nr * xrow,
                              cudaMemcpyHostToDevice, s_in), "H2D chunk");
      RB_CUDA(cudaEventRecord(ev[1 + c], s_in), "event");
      RB_CUDA(cudaStreamWaitEvent(s_cmp, ev[1 + c], 0), "event wait");
      if ((rc = matmul_locked(e, id, xd, x_dtype, nr, k, yd, y_dtype, s_cmp)) != RB_OK) {
        cudaStreamSynchronize(s_in);
        cudaStreamSynchronize(s_cmp);
        cudaStreamSynchronize(s_out);
        return rc;
      }
      RB_CUDA(cudaEventRecord(ev[1 + kHostAttnChunks + c], s_cmp), "event");
      RB_CUDA(cudaStreamWaitEvent(s_out, ev[1 + kHostAttnChunks + c], 0), "event wait");
      RB_CUDA(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(y_host) + r0 * yrow, yd, nr * yrow,
                              cudaMemcpyDeviceToHost, s_out), "D2H chunk");
    }
    RB_CUDA(cudaStreamSynchronize(s_out), "matmul sync");
    RB_CUDA(cudaStreamSynchronize(s_cmp), "matmul sync");
    return RB_OK;
  }
  cudaStream_t st = e->host_stream;
  RB_CUDA(cudaMemcpyAsync(e->io_in.ptr, x_host, xb, cudaMemcpyHostToDevice, st), "H2D");
  if ((rc = matmul_locked(e, id, e->io_in.ptr, x_dtype, m, k, e->io_out.ptr, y_dtype, st)) != RB_OK)
    return rc;
  RB_CUDA(cudaMemcpyAsync(y_host, e->io_out.ptr, yb, cudaMemcpyDeviceToHost, st), "D2H");
  RB_CUDA(cudaStreamSynchronize(st), "matmul sync");
  return RB_OK;
}

int rb_attention(const void* q, const void* k, const void* v, void* out, int dtype, int64_t n_q,
                 int64_t n_kv, int n_head, int n_kv_heads, int head_dim, float scale, float softcap,
                 int mask_mode, int64_t window, int64_t q_start, int64_t kv_start, void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!q || !k || !v || !out) return fail(RB_E_SHAPE, "null attention buffer");
  const int64_t wq = (int64_t)n_head * head_dim, wk = (int64_t)n_kv_heads * head_dim;
  return attention_locked(e, q, wq, k, wk, v, wk, out, wq, dtype, 1, n_q, n_kv, n_head, n_kv_heads,
                          head_dim, scale, softcap, mask_mode, window, q_start, kv_start,
                          reinterpret_cast<cudaStream_t>(stream));
}

int rb_attention_host(const void* q, const void* k, const void* v, void* out, int dtype,
                      int64_t n_q, int64_t n_kv, int n_head, int n_kv_heads, int head_dim,
                      float scale, float softcap, int mask_mode, int64_t window, int64_t q_start,
                      int64_t kv_start) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!q || !k || !v || !out) return fail(RB_E_SHAPE, "null attention buffer");
  const size_t eb = dtype_bytes(dtype);
  if (!eb || n_q <= 0 || n_kv <= 0 || head_dim <= 0 || n_head <= 0 || n_kv_heads <= 0)
    return fail(RB_E_SHAPE, "bad attention arguments");
  const size_t qb = static_cast<size_t>(n_q) * n_head * head_dim * eb;
  const size_t kb = static_cast<size_t>(n_kv) * n_kv_heads * head_dim * eb;
  if ((rc = e->io_in.grow(qb, "q staging")) || (rc = e->io_out.grow(qb, "out staging")) ||
      (rc = e->io_k.grow(kb, "k staging")) || (rc = e->io_v.grow(kb, "v staging")))
    return rc;
  const int64_t wq = (int64_t)n_head * head_dim, wk = (int64_t)n_kv_heads * head_dim;
  // Long full-sequence calls are pipelined: K and V go over first (every
  // query reads all keys), then the query rows in chunks of whole 128-row
  // tiles, each chunk's attention (the same mask as a block mode at the
  // chunk's query offset) starting once its rows are on the device and its
  // output going back while later chunks still copy in or compute. Each
  // row's result is the unchunked call's up to f32 summation order.
  const bool full_seq = mask_mode == RB_MASK_NONE || mask_mode == RB_MASK_CAUSAL ||
                        mask_mode == RB_MASK_WINDOW || mask_mode == RB_MASK_CAUSAL_WINDOW;
  if (full_seq && n_q == n_kv && n_q >= 2048 && dtype != RB_DTYPE_F32) {
    if ((rc = ensure_pipe(e)) != RB_OK) return rc;
    const int block_mode = mask_mode == RB_MASK_NONE     ? RB_MASK_NONE_BLOCK
                           : mask_mode == RB_MASK_WINDOW ? RB_MASK_WINDOW_BLOCK
                                                         : RB_MASK_CAUSAL_BLOCK;
    const int64_t win = mask_mode == RB_MASK_CAUSAL ? -1 : window;
    const int64_t rows = ((n_q + kHostAttnChunks - 1) / kHostAttnChunks + 127) / 128 * 128;
    cudaStream_t s_in = e->pipe_in, s_cmp = e->host_stream, s_out = e->pipe_out;
    cudaEvent_t* ev = e->pipe_ev;  // [0]: K and V in; [1 + c]: chunk c in; [1 + C + c]: chunk c done
    const size_t row_b = static_cast<size_t>(wq) * eb;
    RB_CUDA(cudaMemcpyAsync(e->io_k.ptr, k, kb, cudaMemcpyHostToDevice, s_in), "H2D k");
    RB_CUDA(cudaMemcpyAsync(e->io_v.ptr, v, kb, cudaMemcpyHostToDevice, s_in), "H2D v");
    RB_CUDA(cudaEventRecord(ev[0], s_in), "event");
    RB_CUDA(cudaStreamWaitEvent(s_cmp, ev[0], 0), "event wait");
    int c = 0;
    for (int64_t r0 = 0; r0 < n_q; r0 += rows, ++c) {
      const int64_t nr = n_q - r0 < rows ? n_q - r0 : rows;
      uint8_t* qd = reinterpret_cast<uint8_t*>(e->io_in.ptr) + r0 * row_b;
      uint8_t* od = reinterpret_cast<uint8_t*>(e->io_out.ptr) + r0 * row_b;
      RB_CUDA(cudaMemcpyAsync(qd, reinterpret_cast<const uint8_t*>(q) + r0 * row_b, nr * row_b,
                              cudaMemcpyHostToDevice, s_in), "H2D q chunk");
      RB_CUDA(cudaEventRecord(ev[1 + c], s_in), "event");
      RB_CUDA(cudaStreamWaitEvent(s_cmp, ev[1 + c], 0), "event wait");
      if ((rc = attention_locked(e, qd, wq, e->io_k.ptr, wk, e->io_v.ptr, wk, od, wq, dtype, 1, nr, n_kv,
                                 n_head, n_kv_heads, head_dim, scale, softcap, block_mode, win, r0, 0,
                                 s_cmp)) != RB_OK) {
        cudaStreamSynchronize(s_in);
        cudaStreamSynchronize(s_cmp);
        cudaStreamSynchronize(s_out);
        return rc;
      }
      RB_CUDA(cudaEventRecord(ev[1 + kHostAttnChunks + c], s_cmp), "event");
      RB_CUDA(cudaStreamWaitEvent(s_out, ev[1 + kHostAttnChunks + c], 0), "event wait");
      RB_CUDA(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(out) + r0 * row_b, od, nr * row_b,
                              cudaMemcpyDeviceToHost, s_out), "D2H out chunk");
    }
    RB_CUDA(cudaStreamSynchronize(s_out), "attention sync");
    RB_CUDA(cudaStreamSynchronize(s_cmp), "attention sync");
    return RB_OK;
  }
  cudaStream_t st = e->host_stream;
  RB_CUDA(cudaMemcpyAsync(e->io_in.ptr, q, qb, cudaMemcpyHostToDevice, st), "H2D q");
  RB_CUDA(cudaMemcpyAsync(e->io_k.ptr, k, kb, cudaMemcpyHostToDevice, st), "H2D k");
  RB_CUDA(cudaMemcpyAsync(e->io_v.ptr, v, kb, cudaMemcpyHostToDevice, st), "H2D v");
  if ((rc = attention_locked(e, e->io_in.ptr, wq, e->io_k.ptr, wk, e->io_v.ptr, wk, e->io_out.ptr, wq,
                             dtype, 1, n_q, n_kv, n_head, n_kv_heads, head_dim, scale, softcap,
                             mask_mode, window, q_start, kv_start, st)) != RB_OK)
    return rc;
  RB_CUDA(cudaMemcpyAsync(out, e->io_out.ptr, qb, cudaMemcpyDeviceToHost, st), "D2H out");
  RB_CUDA(cudaStreamSynchronize(st), "attention sync");
  return RB_OK;
}

int rb_attention_batched(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                         int64_t ldv, void* out, int64_t ldo, int dtype, int64_t batch, int64_t n_q,
                         int64_t n_kv, int n_head, int n_kv_heads, int head_dim, float scale,
                         float softcap, int mask_mode, int64_t window, int64_t q_start,
                         int64_t kv_start, void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!q || !k || !v || !out) return fail(RB_E_SHAPE, "null attention buffer");
  return attention_locked(e, q, ldq, k, ldk, v, ldv, out, ldo, dtype, batch, n_q, n_kv, n_head,
                          n_kv_heads, head_dim, scale, softcap, mask_mode, window, q_start, kv_start,
                          reinterpret_cast<cudaStream_t>(stream));
}

// ---- glue
static bool valid_dtype(int dt) { return dt >= RB_DTYPE_F32 && dt <= RB_DTYPE_BF16; }

int rb_rms_norm(const void* x, int x_dtype, const float* w, float eps, void* y, int y_dtype,
                int64_t rows, int64_t d, void* stream) {
  if (!x || !y || rows <= 0 || d <= 0 || !valid_dtype(x_dtype) || !valid_dtype(y_dtype))
    return fail(RB_E_SHAPE, "rms_norm: bad arguments");
  const int rc = launch_rms_norm(x, x_dtype, w, eps, y, y_dtype, rows, static_cast<int>(d),
                                 reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "rms_norm launch failed");
}

static int gated_entry(int act, const void* gate, const void* up, int dtype, void* out, int64_t count,
                       void* stream) {
  if (!gate || !up || !out || count <= 0 || !valid_dtype(dtype))
    return fail(RB_E_SHAPE, "gated activation: bad arguments");
  const int rc = launch_gated(act, gate, up, dtype, count, count, out, dtype, count, 1, count,
                              reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "gated activation launch failed");
}

int rb_silu_mul(const void* gate, const void* up, int dtype, void* out, int64_t count, void* stream) {
  return gated_entry(0, gate, up, dtype, out, count, stream);
}

int rb_gelu_mul(const void* gate, const void* up, int dtype, void* out, int64_t count, void* stream) {
  return gated_entry(1, gate, up, dtype, out, count, stream);
}

int rb_rope(const void* x, int dtype, const float* cos_t, const float* sin_t, void* y, int64_t batch,
            int64_t seq, int heads, int head_dim, void* stream) {
  if (!x || !y || !cos_t || !sin_t || batch <= 0 || seq <= 0 || heads <= 0 || head_dim <= 0 ||
      head_dim % 2 || !valid_dtype(dtype))
    return fail(RB_E_SHAPE, "rope: bad arguments (x must be [B, S, H, D], D even)");
  const int rc = launch_rope(x, dtype, cos_t, sin_t, y, batch * seq, heads, head_dim,
                             static_cast<int>(seq), reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "rope launch failed");
}

int rb_embed_gather(const int32_t* ids, int64_t tokens, const void* table_f16, int64_t vocab, int64_t d,
                    float* x, void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!ids || !table_f16 || !x || tokens <= 0 || vocab <= 0 || d <= 0 || d % 8)
    return fail(RB_E_SHAPE, "embed_gather: bad arguments");
  rc = launch_embed_gather(ids, table_f16, vocab, static_cast<int>(d), x, tokens, e->err,
                           reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "embed_gather launch failed");
}

int rb_add_rms_norm(float* x, const void* delta_f16, const float* w, float eps, void* h_f16,
                    int64_t rows, int64_t d, void* stream) {
  if (!x || !w || !h_f16 || rows <= 0) return fail(RB_E_SHAPE, "add_rms_norm: bad arguments");
  const int rc = launch_add_rms_norm(x, delta_f16, w, eps, h_f16, rows, static_cast<int>(d),
                                     reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "add_rms_norm: unsupported width %lld", (long long)d);
}

int rb_add_layer_norm(float* x, const void* delta_f16, const float* g, const float* b, float eps,
                      void* h_f16, int64_t rows, int64_t d, void* stream) {
  if (!x || !g || !b || !h_f16 || rows <= 0) return fail(RB_E_SHAPE, "add_layer_norm: bad arguments");
  const int rc = launch_add_layer_norm(x, delta_f16, g, b, eps, h_f16, rows, static_cast<int>(d),
                                       reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "add_layer_norm: unsupported width %lld", (long long)d);
}

int rb_gelu(void* y_f16, int64_t count, void* stream) {
  if (!y_f16 || count <= 0) return fail(RB_E_SHAPE, "gelu: bad arguments");
  const int rc = launch_gelu_f16(y_f16, count, reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "gelu: count must be a multiple of 8");
}

int rb_qk_norm_rope(void* qkv_f16, int64_t ld, int64_t tokens, int n_q_heads, int n_kv_heads,
                    int head_dim, const float* q_norm_w, const float* k_norm_w, float eps,
                    const float* cos_t, const float* sin_t, int64_t seq, void* stream) {
  if (!qkv_f16 || !q_norm_w || !k_norm_w || !cos_t || !sin_t || tokens <= 0 || seq <= 0)
    return fail(RB_E_SHAPE, "qk_norm_rope: bad arguments");
  if (head_dim != 128) return fail(RB_E_UNSUPPORTED, "qk_norm_rope: head_dim %d (supported: 128)", head_dim);
  if (n_q_heads <= 0 || n_kv_heads < 0 || ld < static_cast<int64_t>(n_q_heads + n_kv_heads) * 128)
    return fail(RB_E_SHAPE, "qk_norm_rope: row stride %lld below the q and k columns", static_cast<long long>(ld));
  const int rc = launch_qk_norm_rope(qkv_f16, ld, tokens, n_q_heads, n_kv_heads, q_norm_w, k_norm_w, eps,
                                     cos_t, sin_t, static_cast<int>(seq),
                                     reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "qk_norm_rope launch failed");
}

int rb_silu_mul_halves(const void* gu_f16, int64_t rows, int64_t n, void* out_f16, void* stream) {
  if (!gu_f16 || !out_f16 || rows <= 0 || n <= 0) return fail(RB_E_SHAPE, "silu_mul_halves: bad arguments");
  const int rc = launch_silu_mul_halves_f16(gu_f16, rows, n, out_f16, reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "silu_mul_halves: n must be a multiple of 8");
}

int rb_last_token_l2(const float* x, int64_t batch, int64_t seq, int64_t d, const float* w, float eps,
                     float* out, void* stream) {
  if (!x || !w || !out || batch <= 0 || seq <= 0 || d <= 0) return fail(RB_E_SHAPE, "last_token_l2: bad arguments");
  const int rc = launch_last_token_l2(x, static_cast<int>(d), static_cast<int>(seq), static_cast<int>(batch), w,
                                      eps, out, reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "last_token_l2 launch failed");
}

int rb_q8_0_dequant(int64_t id, void* out, int out_dtype, void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  auto it = e->weights.find(id);
  if (it == e->weights.end() || it->second.kind != RB_WEIGHT_Q8_0)
    return fail(RB_E_SHAPE, "weight id %lld is not a Q8_0 weight", (long long)id);
  if (out_dtype != RB_DTYPE_F32 && out_dtype != RB_DTYPE_F16) return fail(RB_E_SHAPE, "dequant dtype");
  const Weight& w = it->second;
  rc = launch_q8_dequant(w.codes, w.scales, static_cast<int>(w.n), static_cast<int>(w.k),
                         static_cast<int>(w.pitch), out,
                         out_dtype == RB_DTYPE_F16, reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "dequant launch failed");
}

int rb_quantize_rows_i8(const void* x, int x_dtype, int64_t m, int64_t k, int8_t* codes,
                        float* row_scale, void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (m <= 0 || k <= 0 || !x || !codes || !row_scale) return fail(RB_E_SHAPE, "bad quantiser arguments");
  rc = launch_quantize_rows_i8(x, x_dtype, m, k, 0.0f, codes, row_scale,
                               reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "quantiser launch failed");
}

int rb_matmul_i8_acc(int64_t id, const int8_t* codes, int64_t m, int32_t* acc, void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  auto it = e->weights.find(id);
  if (it == e->weights.end() || it->second.kind != RB_WEIGHT_W8A8)
    return fail(RB_E_SHAPE, "weight id %lld is not a W8A8 weight", (long long)id);
  const Weight& w = it->second;
  if (m <= 0 || !codes || !acc) return fail(RB_E_SHAPE, "bad int8 matmul arguments");
  CUtensorMap tmA, tmC;
  if ((rc = make_tmap_2d(&tmA, codes, 1, m, w.k, w.k, 128, 128, 128)) != RB_OK) return rc;
  GemmLaunch L{};
  L.M = static_cast<int>(m);
  L.N = static_cast<int>(w.n);
  L.K = static_cast<int>(w.k);
  L.out = acc;
  L.ldo = static_cast<int>(w.n);
  L.out_dtype = RB_DTYPE_I32;
  L.err = e->err;
  L.num_sms = e->num_sms;
  L.s_col = reinterpret_cast<const float*>(w.scales);
  const bool tstore = output_map(&tmC, acc, RB_DTYPE_I32, m, w.n);
  const GemmPlan plan = gemm_plan(true, L.M, L.N, L.K, e->num_sms);
  rc = launch_w8a8_gemm(L, plan, tmA, w.tm_codes[bn_index(plan.weight_rows())], tstore ? &tmC : nullptr,
                        reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "int8 gemm launch failed");
}

int rb_mem_stats(int64_t* weights_bytes, int64_t* scratch_bytes, int64_t* num_weights) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  int64_t wb = 0;
  for (auto& kv : e->weights) wb += static_cast<int64_t>(kv.second.bytes);
  if (weights_bytes) *weights_bytes = wb;
  if (scratch_bytes)
    *scratch_bytes = static_cast<int64_t>(e->act.bytes + e->rowscale.bytes + e->io_in.bytes +
                                          e->io_out.bytes + e->io_k.bytes + e->io_v.bytes);
  if (num_weights) *num_weights = static_cast<int64_t>(e->weights.size());
  return RB_OK;
}

int64_t rb_moe_workspace_bytes(int64_t tokens, int top_k, int experts) {
  if (tokens <= 0 || top_k <= 0 || experts <= 0) return fail(RB_E_SHAPE, "moe workspace: bad sizes");
  return moe_layout(tokens, top_k, experts).words * 4;
}

int64_t rb_moe_max_rows(int64_t tokens, int top_k, int experts) {
  if (tokens <= 0 || top_k <= 0 || experts <= 0) return fail(RB_E_SHAPE, "moe rows: bad sizes");
  return moe_layout(tokens, top_k, experts).max_rows;
}

int64_t rb_moe_slot_rows_offset(int64_t tokens, int top_k, int experts) {
  if (tokens <= 0 || top_k <= 0 || experts <= 0) return fail(RB_E_SHAPE, "moe layout: bad sizes");
  return moe_layout(tokens, top_k, experts).row_of_slot;
}

int rb_moe_route(const float* logits, int64_t tokens, int experts, int top_k, int normalize, int32_t* ids,
                 float* weights, void* stream) {
  if (!logits || !ids || !weights || tokens <= 0) return fail(RB_E_SHAPE, "moe_route: bad arguments");
  const int rc = launch_moe_route(logits, tokens, experts, top_k, normalize, ids, weights,
                                  reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "moe_route: %d experts, top-%d (supported: experts <= 256, k <= 32)",
                                    experts, top_k);
}

int rb_moe_dispatch(const int32_t* ids, int64_t tokens, int top_k, int experts, const void* x_f16,
                    int64_t hidden, void* workspace, void* x_perm_f16, void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!ids || !x_f16 || !workspace || !x_perm_f16 || tokens <= 0 || top_k <= 0)
    return fail(RB_E_SHAPE, "moe_dispatch: bad arguments");
  if ((reinterpret_cast<uintptr_t>(x_f16) | reinterpret_cast<uintptr_t>(x_perm_f16)) & 15)
    return fail(RB_E_SHAPE, "moe_dispatch: rows must be 16-byte aligned");
  rc = launch_moe_dispatch(ids, tokens, top_k, experts, x_f16, hidden, reinterpret_cast<int32_t*>(workspace),
                           x_perm_f16, e->err, reinterpret_cast<cudaStream_t>(stream));
  g_launches += 4;
  return rc == RB_OK ? RB_OK : fail(rc, "moe_dispatch: experts %d (<= 1024), hidden %lld (multiple of 8)",
                                    experts, (long long)hidden);
}

int rb_matmul_grouped(int64_t id, int experts, const void* x_perm_f16, int64_t max_rows, const void* workspace,
                      int64_t tokens, int top_k, void* y, int y_dtype, void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  auto it = e->weights.find(id);
  if (it == e->weights.end()) return fail(RB_E_SHAPE, "weight id %lld is not packed", (long long)id);
  const Weight& w = it->second;
  if (w.kind != RB_WEIGHT_Q8_0) return fail(RB_E_UNSUPPORTED, "grouped matmul: Q8_0 weights only");
  if (experts <= 0 || w.n % experts) return fail(RB_E_SHAPE, "grouped matmul: weight rows not a multiple of experts");
  const MoeLayout ml = moe_layout(tokens, top_k, experts);
  if (max_rows != ml.max_rows) return fail(RB_E_SHAPE, "grouped matmul: max_rows must be rb_moe_max_rows()");
  if (!x_perm_f16 || !workspace || !y || (y_dtype != RB_DTYPE_F16 && y_dtype != RB_DTYPE_F32))
    return fail(RB_E_SHAPE, "grouped matmul: bad arguments");
  const int64_t n = w.n / experts;  // accumulator columns per expert
  const int64_t n_out = w.gated ? n / 2 : n;
  if (w.gated && (y_dtype != RB_DTYPE_F16 || n % 128 != 0))
    return fail(RB_E_SHAPE, "grouped matmul: a gated weight needs f16 output and 64-aligned expert blocks");
  GemmLaunch L{};
  L.M = static_cast<int>(max_rows);
  L.N = static_cast<int>(n);
  L.K = static_cast<int>(w.k);
  L.out = y;
  L.ldo = static_cast<int>(n_out);
  L.gated = w.gated ? 1 : 0;
  L.out_dtype = y_dtype;
  L.err = e->err;
  L.num_sms = e->num_sms;
  L.tile_expert = reinterpret_cast<const int32_t*>(workspace) + ml.tile_expert;
  // CTA-pair tiles (256 rows, one expert: segments are 256-row aligned) when
  // the expert block is a multiple of 128 columns, else single-CTA 128-row
  // tiles; RB_TILES_SINGLE forces the latter.
  const bool pair = n % 128 == 0 && gemm_policy() != RB_TILES_SINGLE;
  const GemmPlan plan = pair ? GemmPlan{n % 256 == 0 ? 256 : 128, 1, true}
                             : GemmPlan{n % 256 == 0 ? 256 : 128, 1, false};
  CUtensorMap tmA, tmC;
  if ((rc = make_tmap_2d(&tmA, x_perm_f16, 2, max_rows, w.k, w.k, 64, 128, 128)) != RB_OK) return rc;
  const bool tstore = output_map(&tmC, y, y_dtype, max_rows, n_out);
  if (w.gated && !tstore) return fail(RB_E_SHAPE, "grouped matmul: output tensor map unavailable");
  const int bi = bn_index(plan.weight_rows());
  L.w_codes = w.codes;
  L.w_scales = w.scales;
  L.w_pitch = w.pitch;
  L.w_rows = w.n;
  if ((rc = launch_q8_gemm(L, plan, tmA, w.tm_codes[bi], w.tm_scales[bi], tstore ? &tmC : nullptr,
                           reinterpret_cast<cudaStream_t>(stream))) != RB_OK)
    return fail(rc, "grouped q8_0 gemm launch failed");
  g_launches++;
  return RB_OK;
}

int rb_moe_combine(float* x, const void* y_perm_f16, int64_t hidden, const int32_t* ids, const float* weights,
                   const void* workspace, int64_t tokens, int top_k, int experts, void* stream) {
  if (!x || !y_perm_f16 || !ids || !weights || !workspace || tokens <= 0)
    return fail(RB_E_SHAPE, "moe_combine: bad arguments");
  const int rc = launch_moe_combine(x, y_perm_f16, hidden, ids, weights, reinterpret_cast<const int32_t*>(workspace),
                                    tokens, top_k, experts, reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "moe_combine: hidden must be a multiple of 8, top_k <= 32");
}

int rb_ep_build_send(const int32_t* ids, int64_t tokens, int top_k, int experts, int ranks, const void* x_f16,
                     int64_t hidden, int32_t* dest_counts, int32_t* dest_cursor, int32_t* send_meta,
                     int32_t* slot_pos, void* send_rows_f16, void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!ids || !x_f16 || !dest_counts || !dest_cursor || !send_meta || !slot_pos || !send_rows_f16 || tokens <= 0)
    return fail(RB_E_SHAPE, "ep_build_send: bad arguments");
  rc = launch_ep_build_send(ids, tokens, top_k, experts, ranks, x_f16, hidden, dest_counts, dest_cursor, send_meta,
                            slot_pos, send_rows_f16, e->err, reinterpret_cast<cudaStream_t>(stream));
  g_launches += 4;
  return rc == RB_OK ? RB_OK : fail(rc, "ep_build_send: experts must divide over ranks, hidden % 8 == 0");
}

int rb_ep_build_send_capacity(const int32_t* ids, int64_t tokens, int top_k, int experts, int ranks,
                              int64_t capacity, const void* x_f16, int64_t hidden, int32_t* dest_counts,
                              int32_t* dest_cursor, int32_t* send_meta, int32_t* slot_pos, void* send_rows_f16,
                              void* stream) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  if (!ids || !x_f16 || !dest_counts || !dest_cursor || !send_meta || !slot_pos || !send_rows_f16 || tokens <= 0 ||
      capacity < 1 || capacity > (1 << 30) / (ranks > 0 ? ranks : 1))
    return fail(RB_E_SHAPE, "ep_build_send_capacity: bad arguments");
  rc = launch_ep_build_send_fixed(ids, tokens, top_k, experts, ranks, static_cast<int>(capacity), x_f16, hidden,
                                  dest_counts, dest_cursor, send_meta, slot_pos, send_rows_f16, e->err,
                                  reinterpret_cast<cudaStream_t>(stream));
  g_launches += 4;
  return rc == RB_OK ? RB_OK : fail(rc, "ep_build_send_capacity: experts must divide over ranks, hidden % 8 == 0");
}

int rb_gather_rows(const void* in_f16, const int32_t* idx, int64_t n, int64_t hidden, void* out_f16, void* stream) {
  if (!in_f16 || !idx || !out_f16 || n < 0) return fail(RB_E_SHAPE, "gather_rows: bad arguments");
  if (n == 0) return RB_OK;
  const int rc = launch_gather_rows(in_f16, idx, n, hidden, out_f16, reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "gather_rows: hidden % 8 == 0");
}

int rb_moe_combine_rows(float* x, const void* y_f16, int64_t hidden, const int32_t* ids, const float* weights,
                        const int32_t* row_of_slot, int64_t tokens, int top_k, void* stream) {
  if (!x || !y_f16 || !ids || !weights || !row_of_slot || tokens <= 0)
    return fail(RB_E_SHAPE, "moe_combine_rows: bad arguments");
  const int rc = launch_moe_combine_rows(x, y_f16, hidden, ids, weights, row_of_slot, tokens, top_k,
                                         reinterpret_cast<cudaStream_t>(stream));
  g_launches++;
  return rc == RB_OK ? RB_OK : fail(rc, "moe_combine_rows: hidden % 8 == 0, top_k <= 32");
}

int rb_set_tile_policy(int policy) {
  if (policy < RB_TILES_AUTO || policy > RB_TILES_PAIR) return fail(RB_E_SHAPE, "unknown tile policy %d", policy);
  return set_gemm_policy(policy);
}

int rb_selftest_wait_timeout(int64_t limit_ns, int64_t* waited_us) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    Engine* e;
    int rc = ensure_engine(&e);
    if (rc) return rc;
    uint32_t* waited = nullptr;
    RB_CUDA(cudaMalloc(&waited, sizeof(uint32_t)), "cudaMalloc(selftest)");
    rc = launch_wait_timeout_probe(e->err, limit_ns, waited, nullptr);
    uint32_t us = 0;
    if (rc == RB_OK) {
      if (cudaDeviceSynchronize() != cudaSuccess ||
          cudaMemcpy(&us, waited, sizeof(us), cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = RB_E_DEVICE;
    }
    cudaFree(waited);
    if (rc) return fail(rc, "wait-timeout probe launch failed (limit %lld ns)", (long long)limit_ns);
    g_launches++;
    if (waited_us) *waited_us = us;
  }
  return rb_check_device_errors();
}

int rb_set_weight_activation(int64_t id, int act) {
  std::lock_guard<std::mutex> lk(g_mu);
  Engine* e;
  int rc = ensure_engine(&e);
  if (rc) return rc;
  auto it = e->weights.find(id);
  if (it == e->weights.end()) return fail(RB_E_SHAPE, "weight id %lld is not packed", (long long)id);
  Weight& w = it->second;
  if (act != RB_ACT_NONE && act != RB_ACT_GELU_TANH) return fail(RB_E_SHAPE, "unknown activation %d", act);
  if (act != RB_ACT_NONE) {
    if (w.gated || w.kind == RB_WEIGHT_I8G)
      return fail(RB_E_SHAPE, "weight id %lld: no fused activation on gated or group-wise weights", (long long)id);
    if (w.kind == RB_WEIGHT_W8A8 && w.out_scale != 0.0f)
      return fail(RB_E_SHAPE, "weight id %lld: no fused activation with a calibrated output grid", (long long)id);
  }
  w.act = act;
  return RB_OK;
}

int rb_set_attention_split(int policy) {
  if (policy < RB_ATTN_SPLIT_AUTO || policy > RB_ATTN_SPLIT_ALWAYS)
    return fail(RB_E_SHAPE, "unknown attention split policy %d", policy);
  return set_attention_split(policy);
}

int64_t rb_launch_count(int reset) {
  return reset ? g_launches.exchange(0) : g_launches.load();
}

}  // extern "C"
