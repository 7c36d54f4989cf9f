// gemm_common.cuh — pieces shared by the single-CTA and CTA-pair tcgen05
// GEMM kernels: launch arguments, Q8_0 dequantisation, and the epilogue that
// turns TMEM accumulators into output tiles.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "sm100.cuh"
#include "kernels.h"

namespace rb {

// Weight kinds of the GEMM kernels: Q8_0 codes dequantised in shared memory
// (kind::f16 UMMA), int8 codes by TMA (kind::i8, W8A8 epilogue), f16 values
// by TMA (kind::f16, the reference's fp16-resident weights).
constexpr int kKindQ8 = 0;
constexpr int kKindI8 = 1;
constexpr int kKindF16 = 2;

constexpr int kEpiWarp0 = 2;      // first epilogue warp
constexpr int kNumEpiWarps = 4;   // Q8_0 kernels: one warp per TMEM lane quarter
constexpr int kNumEpiWarpsI8 = 8; // W8A8 kernels: two warps per lane quarter (column halves)
constexpr int kDqWarp0 = 6;       // first dequant warp (Q8_0 only)
constexpr int kNumDqWarps = 8;
constexpr int kEpiBufBytes = 4096;  // 32 rows x 128 B, one per warp and buffer

enum class BSrc { Tma, Q8Dequant };

constexpr int round1k(int x) { return (x + 1023) & ~1023; }

struct GemmArgs {
  int M, N, K;
  const float* s_row;  // W8A8 [M]
  const float* s_col;  // W8A8 [N]
  void* out;           // [M, ldo]
  int ldo;
  int out_dtype;       // RB_DTYPE_* (RB_DTYPE_I32: raw int8-GEMM accumulators)
  float out_scale;     // W8A8: calibrated output grid (0 = unrounded)
  float out_inv;       // 1 / out_scale in f32
  int epi_path;        // kEpiPath*: how the epilogue writes the output tile
  // Grouped GEMM (MoE experts): per 128-row M tile, the expert whose weight
  // rows [e*N, (e+1)*N) it multiplies, or -1 to skip the tile; nullptr = plain.
  const int* tile_expert;
  // Gated weight (gate and up rows interleaved in blocks of 32): the epilogue
  // writes silu(gate) * up, N/2 f16 columns (kEpiSiluF16).
  int gated;
  // Element-wise activation applied before the f16 rounding (RB_ACT_*).
  int act;
  uint32_t* err;
  int pdl;  // host side: launched with programmatic stream serialization
  // Q8_0 weight in global memory (the CTA-pair kernel's dequant warps read it
  // directly): codes int8 [w_rows, K], scales f16 [K/32, w_pitch].
  const int8_t* w_codes;
  const __half* w_scales;
  long long w_pitch;
  long long w_rows;
};

// Kernel launch, with programmatic stream serialization when `pdl` is set.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t stream, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// --------------------------------------------------------------------------
// Q8_0 dequantisation of 8 consecutive codes of one weight row:
// f16 value = RNE(d * q). 0x6400|u is the f16 number 1024+u, so q = h - 1152
// exactly; one correctly rounded f16 multiply by d then gives RNE(d * q)
// (d * q is exact in f32, so this equals rounding the exact product once).
__device__ __forceinline__ uint4 q8_dequant8_f16(uint2 codes, __half d) {
  const uint32_t lo = codes.x ^ 0x80808080u;
  const uint32_t hi = codes.y ^ 0x80808080u;
  const uint32_t magic = 0x64646464u;
  uint32_t h[4];
  asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(h[0]) : "r"(lo), "r"(magic));
  asm("prmt.b32 %0, %1, %2, 0x7362;" : "=r"(h[1]) : "r"(lo), "r"(magic));
  asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(h[2]) : "r"(hi), "r"(magic));
  asm("prmt.b32 %0, %1, %2, 0x7362;" : "=r"(h[3]) : "r"(hi), "r"(magic));
  const __half2 bias = __half2half2(__ushort_as_half(0x6480));  // 1152.0
  const __half2 d2 = __half2half2(d);
  uint4 out;
  uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 v = *reinterpret_cast<__half2*>(&h[i]);
    v = __hmul2_rn(__hsub2(v, bias), d2);
    o[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return out;
}

// Direct-store fallback: element j of v goes to idx + j when j < count
// (compile-time unrolled so v stays in registers).
__device__ __forceinline__ void store_out16(void* out, int dtype, int64_t idx, const float (&v)[16],
                                            int count) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (j < count) {
      if (dtype == RB_DTYPE_F32 || dtype == RB_DTYPE_I32)  // I32: raw bits in v
        reinterpret_cast<float*>(out)[idx + j] = v[j];
      else if (dtype == RB_DTYPE_F16)
        reinterpret_cast<__half*>(out)[idx + j] = __float2half_rn(v[j]);
      else
        reinterpret_cast<__nv_bfloat16*>(out)[idx + j] = __float2bfloat16_rn(v[j]);
    }
  }
}

// Epilogue parameters held in registers (never through a reference to the
// kernel-parameter struct, which would force a local-memory copy).
struct EpiParams {
  const float* s_col;
  int out_dtype;
  float out_scale, out_inv;
};

// Epilogue value for accumulator bits r at column n (row scale rs).
template <bool I8>
__device__ __forceinline__ float epi_value(const EpiParams e, uint32_t r, float rs, int n) {
  if (!I8) return __uint_as_float(r);
  if (e.out_dtype == RB_DTYPE_I32) return __uint_as_float(r);
  // Order matters for bit parity: f32(acc) * (s_row * s_col).
  float y = __fmul_rn(__int2float_rn(static_cast<int32_t>(r)), __fmul_rn(rs, __ldg(e.s_col + n)));
  if (e.out_scale != 0.0f) {
    // static_code(y, 1/out_scale) * out_scale (ext.rs:1236-1238, 1356-1360),
    // through an integer code like the reference (`as i8`), so zero is +0.0.
    const int code = max(-128, min(127, __float2int_rn(__fmul_rn(y, e.out_inv))));
    y = __fmul_rn(__int2float_rn(code), e.out_scale);
  }
  return y;
}

// Epilogue output paths: element-wise bounds-checked stores (any layout),
// swizzled shared-memory staging + TMA store, or 16-byte vector stores from
// registers (no shared-memory traffic; needs 16-byte aligned rows).
enum : int { kEpiPathScalar = 0, kEpiPathTma = 1, kEpiPathVector = 2 };

// Fast path used when the output allows both (host side; the environment
// variable ROCKET_B200_EPILOGUE=tma|vector overrides the built-in choice).
int epi_path_default();

// Epilogue modes of the TMA-store path, fixed per launch: raw 4-byte
// accumulators (f32 for Q8_0, s32 for RB_DTYPE_I32), f16 / bf16 casts, and the
// W8A8 scaled forms (kEpiS8*; Q = onto the calibrated output grid).
enum : int {
  kEpiRaw4 = 0, kEpiF16, kEpiBF16,
  kEpiS8F32, kEpiS8F16, kEpiS8BF16, kEpiS8F32Q, kEpiS8F16Q, kEpiS8BF16Q,
  kEpiSiluF16,  // gated weight: f16 silu(gate) * up (SwiGLU, host.rs:31-38)
  kEpiF16Gelu, kEpiS8F16Gelu  // f16 gelu_tanh(value) (host.rs:15-18)
};

// gelu_tanh(g) = 0.5 g (1 + tanh(u)), u = sqrt(2/pi) (g + 0.044715 g^3),
// evaluated through the identity 0.5 (1 + tanh(u)) = 1 / (1 + exp(-2u)):
// one exp and one divide, relative error ~1e-6 over the whole range. (A
// tanh approximation with ~2^-11 ABSOLUTE error turns into a large relative
// error in the negative tail, where 1 + tanh(u) is small.) Large negative g:
// exp overflows to +inf and the quotient is -0.
__device__ __forceinline__ float gelu_acc(float g) {
  const float u = (g + g * g * g * 0.044715f) * 0.7978845608028654f;
  return __fdividef(g, 1.0f + __expf(-2.0f * u));
}

// silu on the epilogue path: two MUFU operations (ex2, rcp) per value, so the
// fused epilogue keeps pace with the main loop; a few ulp of f32, far below
// the f16 rounding of the output. Large negative g: exp overflows to +inf
// and the quotient is -0.
__device__ __forceinline__ float silu_acc(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

__host__ __device__ __forceinline__ int epi_mode(bool i8, int out_dtype, float out_scale, int act = 0) {
  if (act == RB_ACT_GELU_TANH) return i8 ? kEpiS8F16Gelu : kEpiF16Gelu;  // f16, no output grid (host checks)
  const int cast = out_dtype == RB_DTYPE_F16 ? 1 : out_dtype == RB_DTYPE_BF16 ? 2 : 0;
  if (!i8 || out_dtype == RB_DTYPE_I32) return out_dtype == RB_DTYPE_I32 ? kEpiRaw4 : cast;
  return kEpiS8F32 + cast + (out_scale != 0.0f ? 3 : 0);
}

// One 32-row x 128-byte chunk of the output tile: this lane's 128 bytes of
// its row go either into the 128-byte-swizzled staging row `b` (for a TMA
// store) or, when `g` is non-null, straight to global memory at `g` as
// 16-byte stores of the groups that lie below column nvalid (`live` = the row
// exists). Columns [0, CW) of the chunk
// from accumulator registers ra (0..31) and rb (32..63, 2-byte outputs only).
// SCALE applies the W8A8 epilogue f32(acc) * (rs * s_col[n]) — in that order,
// for bit parity with ext.rs:1350-1363 — with the chunk's column scales read
// as float4 vectors up front (scp = s_col + first column; nvalid columns are
// in range, the rest clamp to the last valid one and are clipped by the TMA
// store). OUT is the output element size in bytes' role: 4 (f32 / raw), 1 (f16),
// 2 (bf16). QGRID rounds onto the static output grid (ext.rs:1236-1238).
template <bool SCALE, int OUT, bool QGRID, bool GELU = false>
__device__ __forceinline__ void epi_chunk(uint8_t* b, uint4* g, bool live, int lane,
                                          const uint32_t (&ra)[32], const uint32_t (&rb)[32], float rs,
                                          const float* scp, int nvalid, const EpiParams& ep) {
  constexpr int CW = OUT == 4 ? 32 : 64;
  float sc[SCALE ? CW : 1];
  if constexpr (SCALE) {
    if (nvalid >= CW) {
#pragma unroll
      for (int i = 0; i < CW / 4; ++i) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(scp) + i);
        sc[4 * i] = v.x; sc[4 * i + 1] = v.y; sc[4 * i + 2] = v.z; sc[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < CW; ++i) sc[i] = __ldg(scp + min(i, nvalid - 1));
    }
  }
  auto value = [&](int i) -> float {
    const uint32_t r = i < 32 ? ra[i] : rb[i - 32];
    if constexpr (GELU && SCALE) {
      return gelu_acc(__fmul_rn(__int2float_rn(static_cast<int32_t>(r)), __fmul_rn(rs, sc[i])));
    } else if constexpr (GELU) {
      return gelu_acc(__uint_as_float(r));
    } else if constexpr (!SCALE) {
      return __uint_as_float(r);
    } else {
      float y = __fmul_rn(__int2float_rn(static_cast<int32_t>(r)), __fmul_rn(rs, sc[i]));
      if constexpr (QGRID) {
        const int code = max(-128, min(127, __float2int_rn(__fmul_rn(y, ep.out_inv))));
        y = __fmul_rn(__int2float_rn(code), ep.out_scale);
      }
      return y;
    }
  };
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4 o;
    if constexpr (OUT == 4) {
      o = make_uint4(__float_as_uint(value(4 * j)), __float_as_uint(value(4 * j + 1)),
                     __float_as_uint(value(4 * j + 2)), __float_as_uint(value(4 * j + 3)));
    } else {
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float v0 = value(8 * j + 2 * e), v1 = value(8 * j + 2 * e + 1);
        if constexpr (OUT == 1) {
          __half2 h = __floats2half2_rn(v0, v1);
          pk[e] = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
          pk[e] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      o = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    if (g == nullptr) {
      *reinterpret_cast<uint4*>(b + ((j ^ (lane & 7)) << 4)) = o;
    } else if (live && (j + 1) * (CW / 8) <= nvalid) {
      __stcg(g + j, o);  // 16 bytes = CW/8 columns; L2 only (no reuse in L1)
    }
  }
}


// One 128-row block of a finished accumulator (TMEM columns acc_col ..
// acc_col + BN) -> output rows m0 .. m0+127, columns n0 .. n0+BN: each
// epilogue warp owns the TMEM lane quarter `quarter` (32 rows) and the tile
// columns [cbeg, cend). NBUF staging buffers of 4 KB per warp. With
// the TMA path the rows go through this warp's two 4 KB swizzled staging
// buffers (ebuf, alternating by `buf`) and TMA stores clip at the tensor
// edge; the vector path stores each lane's row straight from registers; the
// scalar path stores element by element with bounds checks.
template <int BN, bool I8, int NBUF>
__device__ __forceinline__ void epi_block(uint32_t tmem_base, uint32_t acc_col, int quarter, int lane,
                                          int m0, int n0, int cbeg, int cend, int M, int N,
                                          const float* s_row, void* out, int ldo, int mode,
                                          const EpiParams ep, int path, const CUtensorMap* tmC,
                                          uint8_t* ebuf, int& buf) {
  const bool tma_store = path == kEpiPathTma;
  const bool vec_store = path == kEpiPathVector;
  const int row = quarter * 32 + lane;
  const int CW = (mode == kEpiRaw4 || mode == kEpiS8F32 || mode == kEpiS8F32Q) ? 32 : 64;  // GELU modes: f16
  const int m = m0 + row;
  float rs = 1.0f;
  // Raw int32 output (RB_DTYPE_I32) carries no scales.
  if (I8 && m < M && ep.out_dtype != RB_DTYPE_I32) rs = s_row[m];
  const bool rows_live = m0 + quarter * 32 < M;  // warp-uniform
  if (mode == kEpiSiluF16) {
    // Accumulator columns come in 64-wide groups: 32 gate columns, then the
    // 32 up columns of the same intermediate units. Two groups (128
    // accumulator columns) make one 64-column f16 output chunk at output
    // column (n0 + c0) / 2. TMA-store path only (the host checks).
    if (!rows_live) return;
    for (int c0 = cbeg; c0 < cend && n0 + c0 < N; c0 += 128) {
      if (lane == 0) bulk_wait_read<NBUF - 1>();
      __syncwarp();
      uint8_t* b = ebuf + buf * kEpiBufBytes + lane * 128;
#pragma unroll 1
      for (int hq = 0; hq < 4; ++hq) {  // 16 outputs at a time
        const int cg = c0 + 64 * (hq >> 1) + 16 * (hq & 1);  // gate columns [cg, cg + 16), up at cg + 32
        uint32_t gr[16], ur[16];
        tmem_ld16(tmem_addr(tmem_base, quarter * 32, acc_col + cg), gr);
        tmem_ld16(tmem_addr(tmem_base, quarter * 32, acc_col + cg + 32), ur);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = 8 * j + 2 * e;
            const float v0 = silu_acc(__uint_as_float(gr[i])) * __uint_as_float(ur[i]);
            const float v1 = silu_acc(__uint_as_float(gr[i + 1])) * __uint_as_float(ur[i + 1]);
            __half2 h2 = __floats2half2_rn(v0, v1);
            pk[e] = *reinterpret_cast<uint32_t*>(&h2);
          }
          const int q = 2 * hq + j;  // 16-byte unit of the 128-byte output row
          *reinterpret_cast<uint4*>(b + ((q ^ (lane & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmC, ebuf + buf * kEpiBufBytes, (n0 + c0) / 2, m0 + quarter * 32);
        bulk_commit();
      }
      if (NBUF == 2) buf ^= 1;
    }
    return;
  }
  if (tma_store || vec_store) {
    if (rows_live) {
      for (int c0 = cbeg; c0 < cend && n0 + c0 < N; c0 += CW) {
        uint32_t ra[32], rb[32];  // columns c0..c0+31 and (2-byte outputs) c0+32..c0+63
        tmem_ld32(tmem_addr(tmem_base, quarter * 32, acc_col + c0), ra);
        if (CW == 64) tmem_ld32(tmem_addr(tmem_base, quarter * 32, acc_col + c0 + 32), rb);
        tmem_wait_ld();
        // The buffer about to be written must have been read by its
        // previous TMA store (at most one store of this warp in flight).
        if (tma_store) {
          if (lane == 0) bulk_wait_read<NBUF - 1>();
          __syncwarp();
        }
        uint8_t* b = ebuf + buf * kEpiBufBytes + lane * 128;
        uint4* g = nullptr;
        if (vec_store)
          g = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(out) +
                                       (static_cast<int64_t>(min(m, M - 1)) * ldo + n0 + c0) *
                                           (CW == 64 ? 2 : 4));
        const float* scp = I8 ? ep.s_col + n0 + c0 : nullptr;
        const int nvalid = N - (n0 + c0);
        switch (mode) {
          case kEpiRaw4: epi_chunk<false, 4, false>(b, g, m < M, lane, ra, rb, rs, scp, nvalid, ep); break;
          case kEpiF16: epi_chunk<false, 1, false>(b, g, m < M, lane, ra, rb, rs, scp, nvalid, ep); break;
          case kEpiBF16: epi_chunk<false, 2, false>(b, g, m < M, lane, ra, rb, rs, scp, nvalid, ep); break;
          case kEpiF16Gelu: epi_chunk<false, 1, false, true>(b, g, m < M, lane, ra, rb, rs, scp, nvalid, ep); break;
          default:
            if constexpr (I8) {
              switch (mode) {
                case kEpiS8F32: epi_chunk<true, 4, false>(b, g, m < M, lane, ra, rb, rs, scp, nvalid, ep); break;
                case kEpiS8F16: epi_chunk<true, 1, false>(b, g, m < M, lane, ra, rb, rs, scp, nvalid, ep); break;
                case kEpiS8BF16: epi_chunk<true, 2, false>(b, g, m < M, lane, ra, rb, rs, scp, nvalid, ep); break;
                case kEpiS8F32Q: epi_chunk<true, 4, true>(b, g, m < M, lane, ra, rb, rs, scp, nvalid, ep); break;
                case kEpiS8F16Q: epi_chunk<true, 1, true>(b, g, m < M, lane, ra, rb, rs, scp, nvalid, ep); break;
                case kEpiS8F16Gelu:
                  epi_chunk<true, 1, false, true>(b, g, m < M, lane, ra, rb, rs, scp, nvalid, ep);
                  break;
                default: epi_chunk<true, 2, true>(b, g, m < M, lane, ra, rb, rs, scp, nvalid, ep); break;
              }
            }
            break;
        }
        if (tma_store) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(tmC, ebuf + buf * kEpiBufBytes, n0 + c0, m0 + quarter * 32);
            bulk_commit();
          }
          if (NBUF == 2) buf ^= 1;
        }
      }
    }
  } else {
#pragma unroll 1
    for (int c = cbeg; c < cend; c += 16) {
      uint32_t r[16];
      tmem_ld16(tmem_addr(tmem_base, quarter * 32, acc_col + c), r);
      tmem_wait_ld();
      if (m < M && n0 + c < N) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = epi_value<I8>(ep, r[j], rs, min(n0 + c + j, N - 1));
        const int64_t base = static_cast<int64_t>(m) * ldo + n0 + c;
        store_out16(out, ep.out_dtype, base, v, N - (n0 + c));
      }
    }
  }
}

}  // namespace rb
