// glue.cu — the elementwise / normalisation ops around the matmuls.
//
// RocketOps glue surface (crates/burn-rocket/src/ext.rs:70-83, host formulas
// in crates/burn-rocket/src/host.rs:15-72):
//   rms_norm        x * (mean(x^2) + eps)^-0.5 * w          (host.rs:42-56)
//   silu_mul        g * sigmoid(g) * u, sigmoid = 1/(1+exp(-g))  (host.rs:31-38)
//   gelu_mul        0.5 g (1 + tanh(sqrt(2/pi)(g + 0.044715 g^3))) * u  (host.rs:15-27)
//   rope            rotate-half with [S, D/2] cos/sin tables  (host.rs:61-72)
// and the fused steps of the embedding-model forward:
//   embed_gather    token ids -> f32 rows of an f16 table
//   add_rms_norm    x += delta (f16); h = rms_norm(x) as f16  (residual + norm in one pass)
//   qk_norm_rope    per-head RMSNorm then RoPE, in place on the q and k columns of a fused
//                   q|k|v projection (src/qwen3_embedding/model.rs:355-381)
//   last_token_l2   final RMSNorm of each sequence's last token, L2-normalised
// One warp per row; f32 arithmetic; reductions are warp trees (the reference
// sums sequentially, so sums agree to f32 rounding, not bit for bit).
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "kernels.h"

namespace rb {

__device__ __forceinline__ float ld_f(const void* p, int dt, int64_t i) {
  if (dt == RB_DTYPE_F32) return reinterpret_cast<const float*>(p)[i];
  if (dt == RB_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
__device__ __forceinline__ void st_f(void* p, int dt, int64_t i, float v) {
  if (dt == RB_DTYPE_F32) reinterpret_cast<float*>(p)[i] = v;
  else if (dt == RB_DTYPE_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

static int grid_for_rows(int64_t rows, int warps_per_block) {
  int64_t g = (rows + warps_per_block - 1) / warps_per_block;
  if (g > 148 * 64) g = 148 * 64;
  return static_cast<int>(g < 1 ? 1 : g);
}

// ---------------------------------------------------------------- rms_norm
// Generic: one warp per row of length d; w may be null (scale-free form).
__global__ void rms_norm_kernel(const void* x, int xdt, const float* w, float eps, void* y, int ydt,
                                int64_t rows, int d) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
    const int64_t base = r * d;
    float ss = 0.0f;
    for (int i = lane; i < d; i += 32) {
      const float v = ld_f(x, xdt, base + i);
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(d) + eps);
    for (int i = lane; i < d; i += 32) {
      const float v = ld_f(x, xdt, base + i) * inv;
      st_f(y, ydt, base + i, w ? v * w[i] : v);
    }
  }
}

// ---------------------------------------------------------------- gated activations
__device__ __forceinline__ float silu_f(float g) { return g * (1.0f / (1.0f + expf(-g))); }
__device__ __forceinline__ float gelu_tanh_f(float g) {
  // sqrt(2/pi) as the f32 rounding of the f64 constant (host.rs:10-18).
  const float k = 0.7978845608028654f;
  const float inner = (g + g * g * g * 0.044715f) * k;
  return (g * (tanhf(inner) + 1.0f)) * 0.5f;
}

// out[r, c] = act(a[r, c]) * b[r, c]; a and b may be two halves of one row
// (lda / ldb strides), out has stride ldo.
template <int ACT>
__global__ void gated_kernel(const void* a, const void* b, int dt, int64_t lda, int64_t ldb,
                             void* out, int odt, int64_t ldo, int64_t rows, int64_t cols) {
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const float g = ld_f(a, dt, r * lda + c);
    const float u = ld_f(b, dt, r * ldb + c);
    const float v = ACT == 0 ? silu_f(g) * u : gelu_tanh_f(g) * u;
    st_f(out, odt, r * ldo + c, v);
  }
}

// f16 fast path for silu(gate) * up over the two halves of a gate|up row:
// 8 elements per thread, 16-byte loads and stores.
__global__ void silu_mul_halves_f16_kernel(const __half* gu, int64_t rows, int64_t n, __half* out) {
  const int64_t n8 = n / 8;
  const int64_t total = rows * n8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / n8, c = (i % n8) * 8;
    const uint4 g4 = *reinterpret_cast<const uint4*>(gu + r * 2 * n + c);
    const uint4 u4 = *reinterpret_cast<const uint4*>(gu + r * 2 * n + n + c);
    const __half2* g2 = reinterpret_cast<const __half2*>(&g4);
    const __half2* u2 = reinterpret_cast<const __half2*>(&u4);
    uint4 o4;
    __half2* o2 = reinterpret_cast<__half2*>(&o4);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 g = __half22float2(g2[j]);
      const float2 u = __half22float2(u2[j]);
      o2[j] = __floats2half2_rn(silu_f(g.x) * u.x, silu_f(g.y) * u.y);
    }
    *reinterpret_cast<uint4*>(out + r * n + c) = o4;
  }
}

// ---------------------------------------------------------------- rope
// x [rows, heads, d] (any float dtype, in place allowed); row r uses table row
// pos = (r / heads) % seq. out[j] = x[j] c - x[j+h] s ; out[j+h] = x[j+h] c + x[j] s.
__global__ void rope_kernel(const void* x, int dt, const float* cos_t, const float* sin_t, void* y,
                            int64_t rows, int heads, int d, int seq) {
  const int half = d / 2;
  const int64_t total = rows * heads * half;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t rh = i / half;
    const int j = static_cast<int>(i % half);
    const int64_t r = rh / heads;
    const int pos = static_cast<int>(r % seq);
    const int64_t base = rh * d;
    const float x1 = ld_f(x, dt, base + j), x2 = ld_f(x, dt, base + half + j);
    const float c = cos_t[pos * half + j], s = sin_t[pos * half + j];
    st_f(y, dt, base + j, x1 * c - x2 * s);
    st_f(y, dt, base + half + j, x2 * c + x1 * s);
  }
}

// ---------------------------------------------------------------- fused forward steps
// ids [T] -> x [T, d] f32 from an f16 table [vocab, d].
__global__ void embed_gather_kernel(const int32_t* ids, const __half* table, int64_t vocab, int d,
                                    float* x, int64_t rows, uint32_t* err) {
  const int64_t total = rows * (d / 8);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / (d / 8), c = (i % (d / 8)) * 8;
    int64_t id = ids[r];
    if (id < 0 || id >= vocab) {
      atomicOr(err, 4u);  // kErrBadShape: token id outside the vocabulary
      id = 0;
    }
    const uint4 h4 = *reinterpret_cast<const uint4*>(table + id * d + c);
    const __half2* h2 = reinterpret_cast<const __half2*>(&h4);
    float4 a, b;
    float2 t;
    t = __half22float2(h2[0]); a.x = t.x; a.y = t.y;
    t = __half22float2(h2[1]); a.z = t.x; a.w = t.y;
    t = __half22float2(h2[2]); b.x = t.x; b.y = t.y;
    t = __half22float2(h2[3]); b.z = t.x; b.w = t.y;
    float4* dst = reinterpret_cast<float4*>(x + r * d + c);
    dst[0] = a;
    dst[1] = b;
  }
}

// x [rows, D] f32 (+= delta f16 when non-null), then h = rms_norm(x, w) f16.
// One warp per row; D = 32 * 4 * NV (D % 128 == 0), values kept in registers.
// Row r of x (f32, D = 128 * NV; the lane owns the float4 groups at
// j * 128 + 4 * lane) plus the f16 delta when non-null, the sum written back
// to x. All of the row's loads are issued before its first store: the
// compiler cannot prove x and delta distinct, and a store between two loads
// would hold the later load back (one DRAM round trip per group).
template <int NV>
__device__ __forceinline__ void load_row_add(float* x, const __half* delta, int64_t r, int lane,
                                             float4 (&xv)[NV]) {
  constexpr int D = 128 * NV;
#pragma unroll
  for (int j = 0; j < NV; ++j) xv[j] = *reinterpret_cast<const float4*>(x + r * D + j * 128 + lane * 4);
  if (delta) {
    uint2 d2[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) d2[j] = *reinterpret_cast<const uint2*>(delta + r * D + j * 128 + lane * 4);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&d2[j].x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&d2[j].y));
      xv[j].x += a.x; xv[j].y += a.y; xv[j].z += b.x; xv[j].w += b.y;
      *reinterpret_cast<float4*>(x + r * D + j * 128 + lane * 4) = xv[j];
    }
  }
}

template <int NV>
__global__ void add_rms_norm_kernel(float* x, const __half* delta, const float* w, float eps,
                                    __half* h, int64_t rows) {
  constexpr int D = 128 * NV;
  const int lane = threadIdx.x & 31;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
    float4 xv[NV];
    load_row_add<NV>(x, delta, r, lane, xv);
    float v[4 * NV];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      v[4 * j] = xv[j].x; v[4 * j + 1] = xv[j].y; v[4 * j + 2] = xv[j].z; v[4 * j + 3] = xv[j].w;
      ss = fmaf(xv[j].x, xv[j].x, fmaf(xv[j].y, xv[j].y, fmaf(xv[j].z, xv[j].z, fmaf(xv[j].w, xv[j].w, ss))));
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = j * 128 + lane * 4;
      const float4 wv = *reinterpret_cast<const float4*>(w + c);
      const __half2 a = __floats2half2_rn(v[4 * j] * inv * wv.x, v[4 * j + 1] * inv * wv.y);
      const __half2 b = __floats2half2_rn(v[4 * j + 2] * inv * wv.z, v[4 * j + 3] * inv * wv.w);
      uint2 o;
      o.x = *reinterpret_cast<const uint32_t*>(&a);
      o.y = *reinterpret_cast<const uint32_t*>(&b);
      *reinterpret_cast<uint2*>(h + r * D + c) = o;
    }
  }
}

// x [rows, D] f32 (+= delta f16 when non-null), then
// h = (x - mean) / sqrt(var + eps) * g + b as f16 (pre-LayerNorm of the
// SigLIP-style tower; var is the biased mean of squared deviations).
template <int NV>
__global__ void add_layer_norm_kernel(float* x, const __half* delta, const float* g, const float* b,
                                      float eps, __half* h, int64_t rows) {
  constexpr int D = 128 * NV;
  const int lane = threadIdx.x & 31;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
    float4 xv[NV];
    load_row_add<NV>(x, delta, r, lane, xv);
    float v[4 * NV];
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      v[4 * j] = xv[j].x; v[4 * j + 1] = xv[j].y; v[4 * j + 2] = xv[j].z; v[4 * j + 3] = xv[j].w;
      sum += (xv[j].x + xv[j].y) + (xv[j].z + xv[j].w);
    }
    const float mean = warp_sum(sum) / static_cast<float>(D);
    float var = 0.0f;
#pragma unroll
    for (int i = 0; i < 4 * NV; ++i) {
      const float dv = v[i] - mean;
      var = fmaf(dv, dv, var);
    }
    var = warp_sum(var) / static_cast<float>(D);
    const float inv = 1.0f / sqrtf(var + eps);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = j * 128 + lane * 4;
      const float4 gv = *reinterpret_cast<const float4*>(g + c);
      const float4 bv = *reinterpret_cast<const float4*>(b + c);
      const __half2 a = __floats2half2_rn((v[4 * j] - mean) * inv * gv.x + bv.x,
                                          (v[4 * j + 1] - mean) * inv * gv.y + bv.y);
      const __half2 bb = __floats2half2_rn((v[4 * j + 2] - mean) * inv * gv.z + bv.z,
                                           (v[4 * j + 3] - mean) * inv * gv.w + bv.w);
      uint2 o;
      o.x = *reinterpret_cast<const uint32_t*>(&a);
      o.y = *reinterpret_cast<const uint32_t*>(&bb);
      *reinterpret_cast<uint2*>(h + r * D + c) = o;
    }
  }
}

// In place on f16 [count]: y = gelu_tanh(y) (host.rs:15-18), 8 elements per thread.
__global__ void gelu_f16_kernel(__half* y, int64_t count8) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint4 u = *reinterpret_cast<const uint4*>(y + i * 8);
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      h[j] = __floats2half2_rn(gelu_tanh_f(f.x), gelu_tanh_f(f.y));
    }
    *reinterpret_cast<uint4*>(y + i * 8) = u;
  }
}

// In place on qkv [T, ld] f16: heads [0, hq) of width 128 at column 0 (q) use
// wq, heads [hq, hq+hk) (k) use wk. Each half-warp takes one (token, head):
// lane i of the 16 owns elements 4i..4i+3 and 64+4i..64+4i+3 (the rotate-half
// pairs), read and written as 8-byte vectors; the head's sum of squares is
// reduced over the 16 lanes. Every operation is an explicitly rounded f32
// intrinsic, so the result does not depend on the compiler's contraction.
__global__ void qk_norm_rope_kernel(__half* qkv, int64_t ld, int64_t tokens, int hq, int hk,
                                    const float* wq, const float* wk, float eps,
                                    const float* cos_t, const float* sin_t, int seq) {
  const int lane = threadIdx.x & 31;
  const int hl = lane & 15;  // lane within the half-warp
  const int heads = hq + hk;
  const int64_t tasks = tokens * heads;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  // Warp-uniform loop over task pairs (the shuffles below span the warp);
  // a half-warp past the last task computes on zeros and stores nothing.
  for (int64_t pr = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); 2 * pr < tasks;
       pr += nw) {
    const int64_t task = 2 * pr + (lane >> 4);
    const bool live = task < tasks;
    const int64_t t = live ? task / heads : 0;
    const int hd = live ? static_cast<int>(task % heads) : 0;
    const int pos = static_cast<int>(t % seq);
    __half* p = qkv + t * ld + static_cast<int64_t>(hd) * 128;
    const uint2 ua = live ? *reinterpret_cast<const uint2*>(p + 4 * hl) : make_uint2(0u, 0u);
    const uint2 ub = live ? *reinterpret_cast<const uint2*>(p + 64 + 4 * hl) : make_uint2(0u, 0u);
    const float2 a01 = __half22float2(*reinterpret_cast<const __half2*>(&ua.x));
    const float2 a23 = __half22float2(*reinterpret_cast<const __half2*>(&ua.y));
    const float2 b01 = __half22float2(*reinterpret_cast<const __half2*>(&ub.x));
    const float2 b23 = __half22float2(*reinterpret_cast<const __half2*>(&ub.y));
    const float a[4] = {a01.x, a01.y, a23.x, a23.y};
    const float bb[4] = {b01.x, b01.y, b23.x, b23.y};
    float ss = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(a[e], a[e]), __fmul_rn(bb[e], bb[e])));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 0.0078125f), eps)));
    const float* w = hd < hq ? wq : wk;
    const float4 wa = *reinterpret_cast<const float4*>(w + 4 * hl);
    const float4 wb = *reinterpret_cast<const float4*>(w + 64 + 4 * hl);
    const float4 cs = *reinterpret_cast<const float4*>(cos_t + pos * 64 + 4 * hl);
    const float4 sn = *reinterpret_cast<const float4*>(sin_t + pos * 64 + 4 * hl);
    const float wa4[4] = {wa.x, wa.y, wa.z, wa.w}, wb4[4] = {wb.x, wb.y, wb.z, wb.w};
    const float c4[4] = {cs.x, cs.y, cs.z, cs.w}, s4[4] = {sn.x, sn.y, sn.z, sn.w};
    float oa[4], ob[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a0 = __fmul_rn(__fmul_rn(a[e], inv), wa4[e]), b0 = __fmul_rn(__fmul_rn(bb[e], inv), wb4[e]);
      oa[e] = __fsub_rn(__fmul_rn(a0, c4[e]), __fmul_rn(b0, s4[e]));
      ob[e] = __fadd_rn(__fmul_rn(b0, c4[e]), __fmul_rn(a0, s4[e]));
    }
    const __half2 oa01 = __floats2half2_rn(oa[0], oa[1]), oa23 = __floats2half2_rn(oa[2], oa[3]);
    const __half2 ob01 = __floats2half2_rn(ob[0], ob[1]), ob23 = __floats2half2_rn(ob[2], ob[3]);
    if (live) {
      *reinterpret_cast<uint2*>(p + 4 * hl) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&oa01), *reinterpret_cast<const uint32_t*>(&oa23));
      *reinterpret_cast<uint2*>(p + 64 + 4 * hl) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&ob01), *reinterpret_cast<const uint32_t*>(&ob23));
    }
  }
}

// The same per-head RMSNorm + RoPE with one warp per token and 16-byte
// accesses: lane 8g + j holds values 8j..8j+7 of both rotate-halves of head
// 4p + g in pass p, so a pass covers four consecutive heads (1 KB of the row)
// and all NP passes' loads are issued before any arithmetic. Each warp keeps
// NP x 512 B of its row in flight, which the half-warp-per-head form (two
// 8-byte loads per lane, then a dependent reduction) could not: that form ran
// at ~60% of the HBM copy rate. Per head the sum of squares adds each lane's
// 8 (a^2 + b^2) terms in order and then the 8 lanes by a butterfly.
template <int NP>
__global__ void __launch_bounds__(256, 2)
qk_norm_rope_wide_kernel(__half* qkv, int64_t ld, int64_t tokens, int hq, int hk, const float* wq,
                         const float* wk, float eps, const float* cos_t, const float* sin_t, int seq) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 3, j = lane & 7;
  const int heads = hq + hk;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); t < tokens;
       t += nw) {
    __half* row = qkv + t * ld;
    uint4 va[NP], vb[NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const int h = 4 * p + g;
      if (h < heads) {
        va[p] = *reinterpret_cast<const uint4*>(row + h * 128 + 8 * j);
        vb[p] = *reinterpret_cast<const uint4*>(row + h * 128 + 64 + 8 * j);
      } else {
        va[p] = make_uint4(0u, 0u, 0u, 0u);
        vb[p] = va[p];
      }
    }
    const int pos = static_cast<int>(t % seq);
    const float4 c0 = *reinterpret_cast<const float4*>(cos_t + pos * 64 + 8 * j);
    const float4 c1 = *reinterpret_cast<const float4*>(cos_t + pos * 64 + 8 * j + 4);
    const float4 s0 = *reinterpret_cast<const float4*>(sin_t + pos * 64 + 8 * j);
    const float4 s1 = *reinterpret_cast<const float4*>(sin_t + pos * 64 + 8 * j + 4);
    const float c8[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float s8[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const int h = 4 * p + g;
      float a[8], b[8];
      const __half2* ha = reinterpret_cast<const __half2*>(&va[p]);
      const __half2* hb = reinterpret_cast<const __half2*>(&vb[p]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fa = __half22float2(ha[e]), fb = __half22float2(hb[e]);
        a[2 * e] = fa.x; a[2 * e + 1] = fa.y;
        b[2 * e] = fb.x; b[2 * e + 1] = fb.y;
      }
      float ss = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(a[e], a[e]), __fmul_rn(b[e], b[e])));
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 0.0078125f), eps)));
      const float* w = h < hq ? wq : wk;
      const float4 wa0 = *reinterpret_cast<const float4*>(w + 8 * j);
      const float4 wa1 = *reinterpret_cast<const float4*>(w + 8 * j + 4);
      const float4 wb0 = *reinterpret_cast<const float4*>(w + 64 + 8 * j);
      const float4 wb1 = *reinterpret_cast<const float4*>(w + 64 + 8 * j + 4);
      const float wa8[8] = {wa0.x, wa0.y, wa0.z, wa0.w, wa1.x, wa1.y, wa1.z, wa1.w};
      const float wb8[8] = {wb0.x, wb0.y, wb0.z, wb0.w, wb1.x, wb1.y, wb1.z, wb1.w};
      uint4 oa, ob;
      __half2* pa = reinterpret_cast<__half2*>(&oa);
      __half2* pb = reinterpret_cast<__half2*>(&ob);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float ra[2], rb[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int i = 2 * e + u;
          const float a0 = __fmul_rn(__fmul_rn(a[i], inv), wa8[i]), b0 = __fmul_rn(__fmul_rn(b[i], inv), wb8[i]);
          ra[u] = __fsub_rn(__fmul_rn(a0, c8[i]), __fmul_rn(b0, s8[i]));
          rb[u] = __fadd_rn(__fmul_rn(b0, c8[i]), __fmul_rn(a0, s8[i]));
        }
        pa[e] = __floats2half2_rn(ra[0], ra[1]);
        pb[e] = __floats2half2_rn(rb[0], rb[1]);
      }
      if (h < heads) {
        *reinterpret_cast<uint4*>(row + h * 128 + 8 * j) = oa;
        *reinterpret_cast<uint4*>(row + h * 128 + 64 + 8 * j) = ob;
      }
    }
  }
}

// out[b] = l2_normalise(rms_norm(x[b * seq + seq - 1], w)), one warp per sequence.
__global__ void last_token_l2_kernel(const float* x, int d, int seq, int batch, const float* w,
                                     float eps, float* out) {
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (b >= batch) return;
  const float* row = x + (static_cast<int64_t>(b) * seq + seq - 1) * d;
  float ss = 0.0f;
  for (int i = lane; i < d; i += 32) ss = fmaf(row[i], row[i], ss);
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(d) + eps);
  float nn = 0.0f;
  for (int i = lane; i < d; i += 32) {
    const float v = row[i] * inv * w[i];
    nn = fmaf(v, v, nn);
  }
  nn = warp_sum(nn);
  const float inv2 = 1.0f / fmaxf(sqrtf(nn), 1e-12f);
  for (int i = lane; i < d; i += 32) out[static_cast<int64_t>(b) * d + i] = row[i] * inv * w[i] * inv2;
}

// ---------------------------------------------------------------- launchers
#define RB_LAUNCH_OK() (cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE)

int launch_rms_norm(const void* x, int xdt, const float* w, float eps, void* y, int ydt, int64_t rows,
                    int d, cudaStream_t st) {
  rms_norm_kernel<<<grid_for_rows(rows, 8), 256, 0, st>>>(x, xdt, w, eps, y, ydt, rows, d);
  return RB_LAUNCH_OK();
}

int launch_gated(int act, const void* a, const void* b, int dt, int64_t lda, int64_t ldb, void* out,
                 int odt, int64_t ldo, int64_t rows, int64_t cols, cudaStream_t st) {
  int64_t g = (rows * cols + 255) / 256;
  if (g > 148 * 32) g = 148 * 32;
  if (g < 1) g = 1;
  if (act == 0)
    gated_kernel<0><<<static_cast<int>(g), 256, 0, st>>>(a, b, dt, lda, ldb, out, odt, ldo, rows, cols);
  else
    gated_kernel<1><<<static_cast<int>(g), 256, 0, st>>>(a, b, dt, lda, ldb, out, odt, ldo, rows, cols);
  return RB_LAUNCH_OK();
}

int launch_silu_mul_halves_f16(const void* gu, int64_t rows, int64_t n, void* out, cudaStream_t st) {
  if (n % 8) return RB_E_SHAPE;
  int64_t g = (rows * (n / 8) + 255) / 256;
  if (g > 148 * 32) g = 148 * 32;
  if (g < 1) g = 1;
  silu_mul_halves_f16_kernel<<<static_cast<int>(g), 256, 0, st>>>(
      reinterpret_cast<const __half*>(gu), rows, n, reinterpret_cast<__half*>(out));
  return RB_LAUNCH_OK();
}

int launch_rope(const void* x, int dt, const float* cos_t, const float* sin_t, void* y, int64_t rows,
                int heads, int d, int seq, cudaStream_t st) {
  int64_t g = (rows * heads * (d / 2) + 255) / 256;
  if (g > 148 * 32) g = 148 * 32;
  if (g < 1) g = 1;
  rope_kernel<<<static_cast<int>(g), 256, 0, st>>>(x, dt, cos_t, sin_t, y, rows, heads, d, seq);
  return RB_LAUNCH_OK();
}

int launch_embed_gather(const int32_t* ids, const void* table, int64_t vocab, int d, float* x,
                        int64_t rows, uint32_t* err, cudaStream_t st) {
  if (d % 8) return RB_E_SHAPE;
  int64_t g = (rows * (d / 8) + 255) / 256;
  if (g > 148 * 32) g = 148 * 32;
  if (g < 1) g = 1;
  embed_gather_kernel<<<static_cast<int>(g), 256, 0, st>>>(
      ids, reinterpret_cast<const __half*>(table), vocab, d, x, rows, err);
  return RB_LAUNCH_OK();
}

int launch_add_rms_norm(float* x, const void* delta, const float* w, float eps, void* h, int64_t rows,
                        int d, cudaStream_t st) {
  const int grid = grid_for_rows(rows, 8);
  const __half* dl = reinterpret_cast<const __half*>(delta);
  __half* hh = reinterpret_cast<__half*>(h);
  switch (d) {
    case 1024: add_rms_norm_kernel<8><<<grid, 256, 0, st>>>(x, dl, w, eps, hh, rows); break;
    case 2048: add_rms_norm_kernel<16><<<grid, 256, 0, st>>>(x, dl, w, eps, hh, rows); break;
    case 1152: add_rms_norm_kernel<9><<<grid, 256, 0, st>>>(x, dl, w, eps, hh, rows); break;
    default: return RB_E_UNSUPPORTED;
  }
  return RB_LAUNCH_OK();
}

// add_layer_norm_kernel followed by the W8A8 dynamic per-row activation
// quantiser, without the f16 round trip through memory: the normalised row
// is rounded to f16 (the value the separate quantiser would read), then
// s = max(max|h| / 127, 1e-12) and code = clamp(rint(h * (1/s)), -128, 127)
// exactly as quantize_rows_kernel (ext.rs:1236-1238, 1263-1279), so codes and
// scales are bit-identical to layer norm + rb_quantize_rows_i8.
template <int NV>
__global__ void add_layer_norm_quant_kernel(float* x, const __half* delta, const float* g, const float* b,
                                            float eps, int8_t* codes, float* row_scale, int64_t rows) {
  constexpr int D = 128 * NV;
  const int lane = threadIdx.x & 31;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
    float4 xv[NV];
    load_row_add<NV>(x, delta, r, lane, xv);
    float v[4 * NV];
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      v[4 * j] = xv[j].x; v[4 * j + 1] = xv[j].y; v[4 * j + 2] = xv[j].z; v[4 * j + 3] = xv[j].w;
      sum += (xv[j].x + xv[j].y) + (xv[j].z + xv[j].w);
    }
    const float mean = warp_sum(sum) / static_cast<float>(D);
    float var = 0.0f;
#pragma unroll
    for (int i = 0; i < 4 * NV; ++i) {
      const float dv = v[i] - mean;
      var = fmaf(dv, dv, var);
    }
    var = warp_sum(var) / static_cast<float>(D);
    const float inv = 1.0f / sqrtf(var + eps);
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = j * 128 + lane * 4;
      const float4 gv = *reinterpret_cast<const float4*>(g + c);
      const float4 bv = *reinterpret_cast<const float4*>(b + c);
      const float2 a = __half22float2(__floats2half2_rn((v[4 * j] - mean) * inv * gv.x + bv.x,
                                                        (v[4 * j + 1] - mean) * inv * gv.y + bv.y));
      const float2 bb = __half22float2(__floats2half2_rn((v[4 * j + 2] - mean) * inv * gv.z + bv.z,
                                                         (v[4 * j + 3] - mean) * inv * gv.w + bv.w));
      v[4 * j] = a.x; v[4 * j + 1] = a.y; v[4 * j + 2] = bb.x; v[4 * j + 3] = bb.y;
      amax = fmaxf(fmaxf(amax, fmaxf(fabsf(a.x), fabsf(a.y))), fmaxf(fabsf(bb.x), fabsf(bb.y)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
    const float qinv = __fdiv_rn(1.0f, sc);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = j * 128 + lane * 4;
      char4 q;
      q.x = static_cast<signed char>(fminf(fmaxf(rintf(__fmul_rn(v[4 * j], qinv)), -128.f), 127.f));
      q.y = static_cast<signed char>(fminf(fmaxf(rintf(__fmul_rn(v[4 * j + 1], qinv)), -128.f), 127.f));
      q.z = static_cast<signed char>(fminf(fmaxf(rintf(__fmul_rn(v[4 * j + 2], qinv)), -128.f), 127.f));
      q.w = static_cast<signed char>(fminf(fmaxf(rintf(__fmul_rn(v[4 * j + 3], qinv)), -128.f), 127.f));
      *reinterpret_cast<char4*>(codes + r * D + c) = q;
    }
    if (lane == 0) row_scale[r] = sc;
  }
}

int launch_add_layer_norm_quant(float* x, const void* delta, const float* g, const float* b, float eps,
                                int8_t* codes, float* row_scale, int64_t rows, int d, cudaStream_t st) {
  const int grid = grid_for_rows(rows, 8);
  const __half* dl = reinterpret_cast<const __half*>(delta);
  switch (d) {
    case 1152: add_layer_norm_quant_kernel<9><<<grid, 256, 0, st>>>(x, dl, g, b, eps, codes, row_scale, rows); break;
    case 1024: add_layer_norm_quant_kernel<8><<<grid, 256, 0, st>>>(x, dl, g, b, eps, codes, row_scale, rows); break;
    case 768: add_layer_norm_quant_kernel<6><<<grid, 256, 0, st>>>(x, dl, g, b, eps, codes, row_scale, rows); break;
    default: return RB_E_UNSUPPORTED;
  }
  return RB_LAUNCH_OK();
}

int launch_add_layer_norm(float* x, const void* delta, const float* g, const float* b, float eps,
                          void* h, int64_t rows, int d, cudaStream_t st) {
  const int grid = grid_for_rows(rows, 8);
  const __half* dl = reinterpret_cast<const __half*>(delta);
  __half* hh = reinterpret_cast<__half*>(h);
  switch (d) {
    case 1152: add_layer_norm_kernel<9><<<grid, 256, 0, st>>>(x, dl, g, b, eps, hh, rows); break;
    case 1024: add_layer_norm_kernel<8><<<grid, 256, 0, st>>>(x, dl, g, b, eps, hh, rows); break;
    case 768: add_layer_norm_kernel<6><<<grid, 256, 0, st>>>(x, dl, g, b, eps, hh, rows); break;
    default: return RB_E_UNSUPPORTED;
  }
  return RB_LAUNCH_OK();
}

int launch_gelu_f16(void* y, int64_t count, cudaStream_t st) {
  if (count % 8) return RB_E_SHAPE;
  int64_t g = (count / 8 + 255) / 256;
  if (g > 148 * 32) g = 148 * 32;
  if (g < 1) g = 1;
  gelu_f16_kernel<<<static_cast<int>(g), 256, 0, st>>>(reinterpret_cast<__half*>(y), count / 8);
  return RB_LAUNCH_OK();
}

int launch_qk_norm_rope(void* qkv, int64_t ld, int64_t tokens, int hq, int hk, const float* wq,
                        const float* wk, float eps, const float* cos_t, const float* sin_t, int seq,
                        cudaStream_t st) {
  if ((ld % 4) != 0 || (reinterpret_cast<uintptr_t>(qkv) & 7) != 0) return RB_E_SHAPE;  // 8-byte vectors
  const int np = (hq + hk + 3) / 4;
  if ((ld % 8) == 0 && (reinterpret_cast<uintptr_t>(qkv) & 15) == 0 && np <= 9) {  // up to 36 heads per token without spills
    int64_t wb = (tokens + 7) / 8;  // one token per warp, 8 warps per block
    if (wb > 148 * 16) wb = 148 * 16;
    const int b = static_cast<int>(wb);
    __half* q = reinterpret_cast<__half*>(qkv);
#define RB_QKNR(NP)                                                                                  \
  case NP:                                                                                           \
    qk_norm_rope_wide_kernel<NP><<<b, 256, 0, st>>>(q, ld, tokens, hq, hk, wq, wk, eps, cos_t, sin_t, seq); \
    return RB_LAUNCH_OK();
    switch (np) {
      RB_QKNR(1) RB_QKNR(2) RB_QKNR(3) RB_QKNR(4) RB_QKNR(5) RB_QKNR(6) RB_QKNR(7) RB_QKNR(8) RB_QKNR(9)
      default: break;
    }
#undef RB_QKNR
  }
  int64_t blocks = (tokens * (hq + hk) + 15) / 16;  // two tasks per warp, 8 warps per block
  if (blocks > 148 * 64) blocks = 148 * 64;
  if (blocks < 1) blocks = 1;
  qk_norm_rope_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(
      reinterpret_cast<__half*>(qkv), ld, tokens, hq, hk, wq, wk, eps, cos_t, sin_t, seq);
  return RB_LAUNCH_OK();
}

int launch_last_token_l2(const float* x, int d, int seq, int batch, const float* w, float eps,
                         float* out, cudaStream_t st) {
  last_token_l2_kernel<<<(batch + 7) / 8, 256, 0, st>>>(x, d, seq, batch, w, eps, out);
  return RB_LAUNCH_OK();
}

}  // namespace rb
