// quant.cu — codec and quantiser kernels around the GEMMs:
//   * Q8_0 encode (f32 -> codes + f16 block scale), the reference encoder of
//     crates/rocket-npu/src/bin/q8_bench.rs:199-219, bit for bit;
//   * GGUF Q8_0 block unpack (34-byte AoS blocks -> codes / scales planes),
//     src/util/gguf.rs:197-215;
//   * per-row int8 activation quantiser of the W8A8 path,
//     crates/burn-rocket/src/ext.rs:1236-1238 and 1263-1279;
//   * dtype casts (f32/bf16 -> f16 with round-to-nearest-even, like
//     f32_to_f16_par, ext.rs:2144-2156).
// All arithmetic uses explicitly rounded IEEE intrinsics (__fdiv_rn,
// __fmul_rn) so results match the CPU oracle exactly.
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "kernels.h"
#include "sm100.cuh"

namespace rb {

__device__ __forceinline__ float load_as_f32(const void* p, int dtype, int64_t i) {
  if (dtype == RB_DTYPE_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == RB_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

// ---------------------------------------------------------------- Q8_0 encode
// One thread per 32-value block. d = f16(amax / 127); codes are rounded half
// away from zero against the *stored* f16 scale and clamped to [-127, 127].
__global__ void q8_0_encode_kernel(const float* __restrict__ w, int64_t n, int64_t k,
                                   int64_t pitch, int8_t* __restrict__ codes,
                                   uint16_t* __restrict__ scales) {
  const int64_t nblk = k / 32;
  const int64_t total = n * nblk;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < total;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = b / nblk, g = b % nblk;
    const float* seg = w + row * k + g * 32;
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(seg[i]));
    const __half d = __float2half_rn(__fdiv_rn(amax, 127.0f));
    const float scale = __half2float(d);
    const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    int8_t* q = codes + row * k + g * 32;
    for (int i = 0; i < 32; ++i) {
      const float r = roundf(__fmul_rn(seg[i], inv));  // half away from zero
      q[i] = static_cast<int8_t>(fminf(fmaxf(r, -127.0f), 127.0f));
    }
    scales[g * pitch + row] = __half_as_ushort(d);  // k-block-major [K/32, pitch]
  }
}

int launch_q8_0_encode(const float* w, int64_t n, int64_t k, int64_t pitch, int8_t* codes,
                       uint16_t* scales, cudaStream_t stream) {
  const int64_t total = n * (k / 32);
  int64_t blocks = (total + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  if (blocks < 1) blocks = 1;
  q8_0_encode_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(w, n, k, pitch, codes, scales);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

// ---------------------------------------------------------------- GGUF unpack
// Block b of row r holds bytes [0,2) = f16 scale (little endian), [2,34) = codes.
__global__ void q8_0_unpack_kernel(const uint8_t* __restrict__ blocks, int64_t n, int64_t k,
                                   int64_t pitch, int8_t* __restrict__ codes,
                                   uint16_t* __restrict__ scales) {
  const int64_t nblk = k / 32;
  const int64_t total = n * nblk;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < total;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint8_t* src = blocks + b * 34;
    const int64_t row = b / nblk, g = b % nblk;
    scales[g * pitch + row] = static_cast<uint16_t>(src[0] | (src[1] << 8));  // [K/32, pitch]
    int8_t* dst = codes + b * 32;  // rows are contiguous runs of blocks
    for (int i = 0; i < 32; ++i) dst[i] = static_cast<int8_t>(src[2 + i]);
  }
}

int launch_q8_0_unpack_blocks(const uint8_t* blocks, int64_t n, int64_t k, int64_t pitch,
                              int8_t* codes, uint16_t* scales, cudaStream_t stream) {
  const int64_t total = n * (k / 32);
  int64_t grid = (total + 255) / 256;
  if (grid > 65535) grid = 65535;
  if (grid < 1) grid = 1;
  q8_0_unpack_kernel<<<static_cast<int>(grid), 256, 0, stream>>>(blocks, n, k, pitch, codes, scales);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

// ---------------------------------------------------------------- row quantiser
// One warp per row. Dynamic mode (in_scale == 0): s = max(max|x| / 127, 1e-12).
// Static mode: s = in_scale. code = clamp(rint(x * (1/s)), -128, 127).
template <int DT>
__global__ void quantize_rows_kernel(const void* __restrict__ x, int64_t m, int64_t k,
                                     float in_scale, int8_t* __restrict__ codes,
                                     float* __restrict__ row_scale) {
  griddep_launch_dependents();  // the GEMM reading our output may start its prologue
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
       row < m; row += warps_total) {
    const int64_t base = row * k;
    float s = in_scale;
    if (in_scale == 0.0f) {
      float amax = 0.0f;
      for (int64_t i = lane; i < k; i += 32) amax = fmaxf(amax, fabsf(load_as_f32(x, DT, base + i)));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
    }
    const float inv = __fdiv_rn(1.0f, s);
    int8_t* q = codes + base;
    if ((k & 3) == 0) {
      for (int64_t i = lane * 4; i < k; i += 128) {
        char4 c;
        c.x = static_cast<signed char>(fminf(fmaxf(rintf(__fmul_rn(load_as_f32(x, DT, base + i), inv)), -128.f), 127.f));
        c.y = static_cast<signed char>(fminf(fmaxf(rintf(__fmul_rn(load_as_f32(x, DT, base + i + 1), inv)), -128.f), 127.f));
        c.z = static_cast<signed char>(fminf(fmaxf(rintf(__fmul_rn(load_as_f32(x, DT, base + i + 2), inv)), -128.f), 127.f));
        c.w = static_cast<signed char>(fminf(fmaxf(rintf(__fmul_rn(load_as_f32(x, DT, base + i + 3), inv)), -128.f), 127.f));
        *reinterpret_cast<char4*>(q + i) = c;
      }
    } else {
      for (int64_t i = lane; i < k; i += 32)
        q[i] = static_cast<int8_t>(
            fminf(fmaxf(rintf(__fmul_rn(load_as_f32(x, DT, base + i), inv)), -128.f), 127.f));
    }
    if (lane == 0) row_scale[row] = s;
  }
}

// Vectorised form for 16-bit activations with k % 16 == 0 and 16-byte
// aligned rows: 16-byte loads (8 values) and 8-byte code stores, the row read
// twice (the second pass hits L1/L2). Same arithmetic as quantize_rows_kernel,
// so codes and scales are identical.
template <int DT>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (DT == RB_DTYPE_F16) {
      const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      const float2 t = __half22float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    } else {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      const float2 t = __bfloat1622float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
}

// V = 16-byte vectors each lane keeps in registers: the row is read once
// (k <= 2048).
template <int DT, int V>
__global__ void quantize_rows_vec_kernel(const uint4* __restrict__ x, int64_t m, int64_t k,
                                         float in_scale, uint2* __restrict__ codes,
                                         float* __restrict__ row_scale) {
  griddep_launch_dependents();  // the GEMM reading our output may start its prologue
  const int lane = threadIdx.x & 31;
  const int nv = static_cast<int>(k / 8);  // 16-byte vectors per row (<= 32 V)
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
       row < m; row += warps_total) {
    const uint4* xr = x + row * nv;
    uint4 v[V];
#pragma unroll
    for (int i = 0; i < V; ++i)
      if (lane + 32 * i < nv) v[i] = __ldg(xr + lane + 32 * i);
    float s = in_scale;
    if (in_scale == 0.0f) {
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        if (lane + 32 * i < nv) {
          float f[8];
          unpack8<DT>(v[i], f);
#pragma unroll
          for (int q = 0; q < 8; ++q) amax = fmaxf(amax, fabsf(f[q]));
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
    }
    const float inv = __fdiv_rn(1.0f, s);
    uint2* q = codes + row * nv;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      if (lane + 32 * i < nv) {
        float f[8];
        unpack8<DT>(v[i], f);
        uint32_t b[2] = {0u, 0u};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = static_cast<int>(fminf(fmaxf(rintf(__fmul_rn(f[e], inv)), -128.f), 127.f));
          b[e >> 2] |= (static_cast<uint32_t>(c) & 0xFFu) << (8 * (e & 3));
        }
        q[lane + 32 * i] = make_uint2(b[0], b[1]);
      }
    }
    if (lane == 0) row_scale[row] = s;
  }
}

// Rows of 2048 < k <= 1024 * V: one block of four warps per row holds the row
// in registers (V 16-byte vectors a thread), so the row is read once. The
// four warps' maxima meet in shared memory, double-buffered by row parity so
// that one barrier per row suffices (a warp writes row i + 2's slot only
// after every warp has passed row i + 1's barrier, i.e. has read row i's).
template <int DT, int V>
__global__ void __launch_bounds__(128) quantize_rows_block_kernel(const uint4* __restrict__ x, int64_t m,
                                                                   int64_t k, float in_scale,
                                                                   uint2* __restrict__ codes,
                                                                   float* __restrict__ row_scale) {
  griddep_launch_dependents();  // the GEMM reading our output may start its prologue
  __shared__ float s_max[2][4];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int nv = static_cast<int>(k / 8);
  int buf = 0;
  for (int64_t row = blockIdx.x; row < m; row += gridDim.x, buf ^= 1) {
    const uint4* xr = x + row * nv;
    uint4 v[V];
#pragma unroll
    for (int i = 0; i < V; ++i)
      if (t + 128 * i < nv) v[i] = __ldg(xr + t + 128 * i);
    float s = in_scale;
    if (in_scale == 0.0f) {  // uniform over the grid
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        if (t + 128 * i < nv) {
          float f[8];
          unpack8<DT>(v[i], f);
#pragma unroll
          for (int q = 0; q < 8; ++q) amax = fmaxf(amax, fabsf(f[q]));
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0) s_max[buf][warp] = amax;
      __syncthreads();
      amax = fmaxf(fmaxf(s_max[buf][0], s_max[buf][1]), fmaxf(s_max[buf][2], s_max[buf][3]));
      s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
    }
    const float inv = __fdiv_rn(1.0f, s);
    uint2* q = codes + row * nv;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      if (t + 128 * i < nv) {
        float f[8];
        unpack8<DT>(v[i], f);
        uint32_t b[2] = {0u, 0u};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = static_cast<int>(fminf(fmaxf(rintf(__fmul_rn(f[e], inv)), -128.f), 127.f));
          b[e >> 2] |= (static_cast<uint32_t>(c) & 0xFFu) << (8 * (e & 3));
        }
        q[t + 128 * i] = make_uint2(b[0], b[1]);
      }
    }
    if (t == 0) row_scale[row] = s;
  }
}

// Longer rows (k > 8192): stream the row twice instead of holding it (the
// second pass hits L1/L2), keeping registers low and many rows in flight.
template <int DT>
__global__ void quantize_rows_stream_kernel(const uint4* __restrict__ x, int64_t m, int64_t k,
                                            float in_scale, uint2* __restrict__ codes,
                                            float* __restrict__ row_scale) {
  griddep_launch_dependents();  // the GEMM reading our output may start its prologue
  const int lane = threadIdx.x & 31;
  const int64_t nv = k / 8;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
       row < m; row += warps_total) {
    const uint4* xr = x + row * nv;
    float s = in_scale;
    if (in_scale == 0.0f) {
      float amax = 0.0f;
#pragma unroll 4
      for (int64_t i = lane; i < nv; i += 32) {
        float f[8];
        unpack8<DT>(__ldg(xr + i), f);
#pragma unroll
        for (int q = 0; q < 8; ++q) amax = fmaxf(amax, fabsf(f[q]));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
    }
    const float inv = __fdiv_rn(1.0f, s);
    uint2* q = codes + row * nv;
#pragma unroll 4
    for (int64_t i = lane; i < nv; i += 32) {
      float f[8];
      unpack8<DT>(__ldg(xr + i), f);
      uint32_t b[2] = {0u, 0u};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int c = static_cast<int>(fminf(fmaxf(rintf(__fmul_rn(f[e], inv)), -128.f), 127.f));
        b[e >> 2] |= (static_cast<uint32_t>(c) & 0xFFu) << (8 * (e & 3));
      }
      q[i] = make_uint2(b[0], b[1]);
    }
    if (lane == 0) row_scale[row] = s;
  }
}

template <int DT>
static void launch_qrv(const void* x, int64_t m, int64_t k, float in_scale, int8_t* codes, float* row_scale,
                       int blocks, cudaStream_t stream) {
  const int nv = static_cast<int>(k / 8);
  const uint4* xv = static_cast<const uint4*>(x);
  uint2* cv = reinterpret_cast<uint2*>(codes);
  if (nv <= 32 * 4) {
    quantize_rows_vec_kernel<DT, 4><<<blocks, 256, 0, stream>>>(xv, m, k, in_scale, cv, row_scale);
  } else if (nv <= 32 * 8) {
    quantize_rows_vec_kernel<DT, 8><<<blocks, 256, 0, stream>>>(xv, m, k, in_scale, cv, row_scale);
  } else if (nv <= 128 * 8) {
    const int64_t bb = m < 148 * 16 ? m : 148 * 16;
    quantize_rows_block_kernel<DT, 8><<<static_cast<int>(bb), 128, 0, stream>>>(xv, m, k, in_scale, cv, row_scale);
  } else {
    const int sb = blocks < 148 * 8 ? blocks : 148 * 8;
    quantize_rows_stream_kernel<DT><<<sb, 256, 0, stream>>>(xv, m, k, in_scale, cv, row_scale);
  }
}

int launch_quantize_rows_i8(const void* x, int x_dtype, int64_t m, int64_t k, float in_scale,
                            int8_t* codes, float* row_scale, cudaStream_t stream) {
  const bool vec = (x_dtype == RB_DTYPE_F16 || x_dtype == RB_DTYPE_BF16) && k % 8 == 0 &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(codes) & 7) == 0;
  if (vec) {
    // one warp per row; blocks of 8 rows, no grid-stride tail to balance
    int64_t blocks = (m + 7) / 8;
    if (blocks > (1 << 30)) blocks = 1 << 30;
    if (blocks < 1) blocks = 1;
    if (x_dtype == RB_DTYPE_F16)
      launch_qrv<RB_DTYPE_F16>(x, m, k, in_scale, codes, row_scale, static_cast<int>(blocks), stream);
    else
      launch_qrv<RB_DTYPE_BF16>(x, m, k, in_scale, codes, row_scale, static_cast<int>(blocks), stream);
    return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
  }
  const int threads = 256;
  int64_t blocks = (m + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  switch (x_dtype) {
    case RB_DTYPE_F32:
      quantize_rows_kernel<RB_DTYPE_F32><<<static_cast<int>(blocks), threads, 0, stream>>>(
          x, m, k, in_scale, codes, row_scale);
      break;
    case RB_DTYPE_F16:
      quantize_rows_kernel<RB_DTYPE_F16><<<static_cast<int>(blocks), threads, 0, stream>>>(
          x, m, k, in_scale, codes, row_scale);
      break;
    case RB_DTYPE_BF16:
      quantize_rows_kernel<RB_DTYPE_BF16><<<static_cast<int>(blocks), threads, 0, stream>>>(
          x, m, k, in_scale, codes, row_scale);
      break;
    default:
      return RB_E_SHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

// ---------------------------------------------------------------- W8A8 weight codes
// Per output channel (row) of an f32 [n, k] weight: s = max(max|w| / 127, 1e-12),
// code = clamp(rint(w * (1/s)), -127, 127) — symmetric per-channel int8, the
// form of a QAT checkpoint's codes + w_scale that pack_qat takes
// (ext.rs:1382-1425). One warp per row.
__global__ void w8a8_weight_quant_kernel(const float* __restrict__ w, int64_t n, int64_t k,
                                         int8_t* __restrict__ codes, float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); r < n; r += nw) {
    const float* row = w + r * k;
    float amax = 0.0f;
    for (int64_t i = lane; i < k; i += 32) amax = fmaxf(amax, fabsf(row[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
    const float inv = __fdiv_rn(1.0f, s);
    for (int64_t i = lane; i < k; i += 32)
      codes[r * k + i] = static_cast<int8_t>(fminf(fmaxf(rintf(__fmul_rn(row[i], inv)), -127.f), 127.f));
    if (lane == 0) scale[r] = s;
  }
}

int launch_w8a8_weight_quant(const float* w, int64_t n, int64_t k, int8_t* codes, float* scale,
                             cudaStream_t stream) {
  int64_t blocks = (n + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  w8a8_weight_quant_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(w, n, k, codes, scale);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

// ---------------------------------------------------------------- group-wise int8
// Per row and per `group`-wide K block: scale = max(max|x| / 127, 1e-12),
// code = clamp(round_half_away(x * (1/scale)), -127, 127)
// (quantize_row_groups, crates/burn-rocket/src/host.rs:77-90). One warp per
// row; scales [m, k/group].
template <int DT>
__global__ void quantize_groups_kernel(const void* __restrict__ x, int64_t m, int64_t k, int group,
                                       int8_t* __restrict__ codes, float* __restrict__ scales) {
  griddep_launch_dependents();  // the GEMM reading our output may start its prologue
  const int lane = threadIdx.x & 31;
  const int64_t ng = k / group;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); row < m;
       row += nw) {
    const int64_t base = row * k;
    for (int64_t g = 0; g < ng; ++g) {
      const int64_t g0 = base + g * group;
      float amax = 0.0f;
      for (int i = lane; i < group; i += 32) amax = fmaxf(amax, fabsf(load_as_f32(x, DT, g0 + i)));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
      const float inv = __fdiv_rn(1.0f, s);
      for (int i = lane; i < group; i += 32)
        codes[g0 + i] = static_cast<int8_t>(
            fminf(fmaxf(roundf(__fmul_rn(load_as_f32(x, DT, g0 + i), inv)), -127.f), 127.f));
      if (lane == 0) scales[row * ng + g] = s;
    }
  }
}

int launch_quantize_groups(const void* x, int x_dtype, int64_t m, int64_t k, int group, int8_t* codes,
                           float* scales, cudaStream_t st) {
  if (group <= 0 || k % group) return RB_E_SHAPE;
  int64_t blocks = (m + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  switch (x_dtype) {
    case RB_DTYPE_F32:
      quantize_groups_kernel<RB_DTYPE_F32><<<static_cast<int>(blocks), 256, 0, st>>>(x, m, k, group, codes, scales);
      break;
    case RB_DTYPE_F16:
      quantize_groups_kernel<RB_DTYPE_F16><<<static_cast<int>(blocks), 256, 0, st>>>(x, m, k, group, codes, scales);
      break;
    case RB_DTYPE_BF16:
      quantize_groups_kernel<RB_DTYPE_BF16><<<static_cast<int>(blocks), 256, 0, st>>>(x, m, k, group, codes, scales);
      break;
    default:
      return RB_E_SHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

// ---------------------------------------------------------------- casts
template <int SRC, int DST>
__global__ void cast_kernel(const void* __restrict__ x, void* __restrict__ y, int64_t count) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = load_as_f32(x, SRC, i);
    if (DST == RB_DTYPE_F32) reinterpret_cast<float*>(y)[i] = v;
    else if (DST == RB_DTYPE_F16) reinterpret_cast<__half*>(y)[i] = __float2half_rn(v);
    else reinterpret_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v);
  }
}

// f32 -> f16, 8 elements per thread (the hot cast on the Q8_0 matmul path).
__global__ void cast_f32_f16_vec_kernel(const float4* __restrict__ x, uint4* __restrict__ y,
                                        int64_t count8) {
  griddep_launch_dependents();  // the GEMM reading our output may start its prologue
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 a = x[2 * i], b = x[2 * i + 1];
    uint4 o;
    __half2* h = reinterpret_cast<__half2*>(&o);
    h[0] = __floats2half2_rn(a.x, a.y);
    h[1] = __floats2half2_rn(a.z, a.w);
    h[2] = __floats2half2_rn(b.x, b.y);
    h[3] = __floats2half2_rn(b.z, b.w);
    y[i] = o;
  }
}

// The same cast for small inputs (up to 148 x 128 x 4 groups of 8), shaped
// to sit beside the GEMM that consumes it: at most one 128-thread CTA per SM
// and at most 56 registers a thread (__launch_bounds__(128, 9)), so an SM
// running one still has the registers for a CTA-pair GEMM CTA (19 warps x 96),
// which under programmatic dependent launch then sets up and stages its
// weights meanwhile. Each thread converts up to four groups, every load
// issued before the first store.
__global__ void __launch_bounds__(128, 9)
cast_f32_f16_x4_kernel(const float4* __restrict__ x, uint4* __restrict__ y, int64_t count8) {
  griddep_launch_dependents();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t i0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  float4 a[4], b[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t i = i0 + j * stride;
    if (i < count8) {
      a[j] = x[2 * i];
      b[j] = x[2 * i + 1];
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t i = i0 + j * stride;
    if (i < count8) {
      uint4 o;
      __half2* h = reinterpret_cast<__half2*>(&o);
      h[0] = __floats2half2_rn(a[j].x, a[j].y);
      h[1] = __floats2half2_rn(a[j].z, a[j].w);
      h[2] = __floats2half2_rn(b[j].x, b[j].y);
      h[3] = __floats2half2_rn(b[j].z, b[j].w);
      y[i] = o;
    }
  }
}

int launch_cast(const void* x, int x_dtype, void* y, int y_dtype, int64_t count,
                cudaStream_t stream) {
  const int threads = 256;
  if (x_dtype == RB_DTYPE_F32 && y_dtype == RB_DTYPE_F16 && (count & 7) == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    const int64_t c8 = count / 8;
    if (c8 <= 148 * 128 * 4) {
      const int64_t blocks = (c8 + 128 * 4 - 1) / (128 * 4);
      cast_f32_f16_x4_kernel<<<static_cast<int>(blocks), 128, 0, stream>>>(
          reinterpret_cast<const float4*>(x), reinterpret_cast<uint4*>(y), c8);
      return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
    }
    int64_t blocks = (c8 + threads - 1) / threads;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    cast_f32_f16_vec_kernel<<<static_cast<int>(blocks), threads, 0, stream>>>(
        reinterpret_cast<const float4*>(x), reinterpret_cast<uint4*>(y), c8);
    return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
  }
  int64_t blocks = (count + threads - 1) / threads;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  const int g = static_cast<int>(blocks);
#define RB_CAST_CASE(S, D)                                                   \
  if (x_dtype == S && y_dtype == D) {                                        \
    cast_kernel<S, D><<<g, threads, 0, stream>>>(x, y, count);               \
    return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;          \
  }
  RB_CAST_CASE(RB_DTYPE_F32, RB_DTYPE_F16)
  RB_CAST_CASE(RB_DTYPE_F32, RB_DTYPE_BF16)
  RB_CAST_CASE(RB_DTYPE_F16, RB_DTYPE_F32)
  RB_CAST_CASE(RB_DTYPE_BF16, RB_DTYPE_F32)
  RB_CAST_CASE(RB_DTYPE_BF16, RB_DTYPE_F16)
  RB_CAST_CASE(RB_DTYPE_F16, RB_DTYPE_BF16)
#undef RB_CAST_CASE
  return RB_E_SHAPE;
}

}  // namespace rb
