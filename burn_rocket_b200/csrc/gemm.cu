// gemm.cu — persistent tcgen05 GEMMs for the two resident-weight matmul kinds
// burn-rocket offloads:
//
//   * Q8_0:  C[M,N] = A[M,K] (f16) · deq(W)[N,K]^T, deq(W) = f16(d · q) built
//            in shared memory from int8 codes + f16 block scales (blocks of 32
//            along K) by producer warps, feeding kind::f16 UMMA with an f32
//            TMEM accumulator. (Reference semantics: the NPU route packs
//            dequantised Q8_0 as fp16, ext.rs:1437-1499; the Q8_0 codec is
//            util/gguf.rs:197-215.)
//   * W8A8:  acc[M,N] = Aq[M,K] (s8) · Wq[N,K]^T (s8) on kind::i8 UMMA with an
//            s32 TMEM accumulator; epilogue y = f32(acc) · (s_row[m] · s_col[n])
//            in exactly that order (ext.rs:1350-1363).
//
// Warp roles (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer (A always; B too for W8A8)
//   warp 1      UMMA issuer (single elected lane) + TMEM owner
//   warps 2..5  epilogue: TMEM -> registers -> global (one accumulator row per thread)
//   warps 6..13 Q8_0 only: dequantise weight codes into the swizzled B stage
// The accumulator is double-buffered in TMEM so the epilogue of tile i overlaps
// the main loop of tile i+1.
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "sm100.cuh"
#include "kernels.h"

namespace rb {

constexpr int kBM = 128;          // UMMA M (one TMEM lane per output row)
constexpr int kStageBytesK = 128; // bytes of K per stage (one 128-B swizzle atom)
constexpr int kEpiWarp0 = 2;      // first epilogue warp
constexpr int kNumEpiWarps = 4;
constexpr int kDqWarp0 = 6;       // first dequant warp (Q8_0 only)
constexpr int kNumDqWarps = 8;

enum class BSrc { Tma, Q8Dequant };

template <int BN_, int STAGES_, bool I8_, BSrc BSRC_>
struct GemmCfg {
  static constexpr int BN = BN_;
  static constexpr int STAGES = STAGES_;
  static constexpr bool I8 = I8_;
  static constexpr BSrc B_SRC = BSRC_;
  static constexpr int ELEM = I8 ? 1 : 2;                   // operand bytes
  static constexpr int BK = kStageBytesK / ELEM;             // K elements per stage
  static constexpr int UMMA_K = I8 ? 32 : 16;                // K per instruction
  static constexpr int KSTEPS = BK / UMMA_K;                 // 4
  static constexpr int A_BYTES = kBM * kStageBytesK;         // 16 KB
  static constexpr int B_BYTES = BN * kStageBytesK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NUM_WARPS = (B_SRC == BSrc::Q8Dequant) ? (kDqWarp0 + kNumDqWarps) : 6;
  static constexpr int THREADS = NUM_WARPS * 32;
  static constexpr uint32_t TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64
                                        : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(2 * BN <= 512, "two accumulators must fit in TMEM");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N constraint for M=128");
};

struct GemmArgs {
  int M, N, K;
  // Q8_0 weight planes (unused for W8A8)
  const int8_t* w_codes;   // [N, K]
  const __half* w_scales;  // [N, K/32]
  // W8A8 scales (unused for Q8_0)
  const float* s_row;      // [M]
  const float* s_col;      // [N]
  void* out;               // [M, ldo]
  int ldo;
  int out_dtype;           // RB_DTYPE_* (RB_DTYPE_I32: raw int8-GEMM accumulators)
  float out_scale;         // W8A8: calibrated output grid (0 = unrounded)
  float out_inv;           // 1 / out_scale in f32
  uint32_t* err;
};

// --------------------------------------------------------------------------
// Q8_0 dequantisation of 8 consecutive codes of one weight row:
// f16 value = RNE(d * q), computed as (biased-exponent trick: 0x6400|u is the
// f16 number 1024+u) q = h - 1152 exactly, then one correctly rounded f16
// multiply by the block scale d.
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

__device__ __forceinline__ void store_out8(void* out, int dtype, int64_t idx, const float* v,
                                           int count) {
  if (dtype == RB_DTYPE_F32 || dtype == RB_DTYPE_I32) {  // I32: raw bits in v
    float* p = reinterpret_cast<float*>(out) + idx;
    if (count == 8 && (idx & 3) == 0) {
      reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      for (int i = 0; i < count; ++i) p[i] = v[i];
    }
  } else if (dtype == RB_DTYPE_F16) {
    __half* p = reinterpret_cast<__half*>(out) + idx;
    if (count == 8 && (idx & 7) == 0) {
      uint4 u;
      __half2* h = reinterpret_cast<__half2*>(&u);
      for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      *reinterpret_cast<uint4*>(p) = u;
    } else {
      for (int i = 0; i < count; ++i) p[i] = __float2half_rn(v[i]);
    }
  } else {
    __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(out) + idx;
    if (count == 8 && (idx & 7) == 0) {
      uint4 u;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
      for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      *reinterpret_cast<uint4*>(p) = u;
    } else {
      for (int i = 0; i < count; ++i) p[i] = __float2bfloat16_rn(v[i]);
    }
  }
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            GemmArgs args) {
  constexpr int BN = Cfg::BN;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128-B swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* full_a = bars;                 // [STAGES] TMA bytes (A, and B for W8A8)
  uint64_t* full_b = bars + STAGES;        // [STAGES] dequant warps (Q8_0)
  uint64_t* empty = bars + 2 * STAGES;     // [STAGES] UMMA commit
  uint64_t* acc_full = bars + 3 * STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = args.M, N = args.N, K = args.K;
  const int tiles_n = (N + BN - 1) / BN;
  const int tiles_m = (M + kBM - 1) / kBM;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + Cfg::BK - 1) / Cfg::BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&full_b[s], kNumDqWarps);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kNumEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    if (Cfg::B_SRC == BSrc::Tma) tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one_sync()) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        const int m0 = (t / tiles_n) * kBM;
        const int n0 = (t % tiles_n) * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, args.err, abort_flag)) goto producer_done;
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          if (Cfg::B_SRC == BSrc::Tma) {
            mbar_arrive_expect_tx(&full_a[stage], Cfg::A_BYTES + Cfg::B_BYTES);
            tma_load_2d(sa, &tmA, &full_a[stage], kb * Cfg::BK, m0);
            tma_load_2d(sa + Cfg::A_BYTES, &tmB, &full_a[stage], kb * Cfg::BK, n0);
          } else {
            mbar_arrive_expect_tx(&full_a[stage], Cfg::A_BYTES);
            tma_load_2d(sa, &tmA, &full_a[stage], kb * Cfg::BK, m0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t idesc =
          Cfg::I8 ? idesc_i8(kBM, BN) : idesc_f16(kBM, BN, false, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, args.err, abort_flag)) goto mma_done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_a[stage], phase, args.err, abort_flag)) goto mma_done;
          if (Cfg::B_SRC == BSrc::Q8Dequant) {
            if (!mbar_wait(&full_b[stage], phase, args.err, abort_flag)) goto mma_done;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t b_addr = a_addr + Cfg::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < Cfg::KSTEPS; ++ks) {
            const uint64_t da = desc_kmajor_sw128(a_addr + ks * 32);
            const uint64_t db = desc_kmajor_sw128(b_addr + ks * 32);
            const uint32_t accum = (kb > 0 || ks > 0) ? 1u : 0u;
            if (Cfg::I8) umma_i8_ss(d_tmem, da, db, idesc, accum);
            else umma_f16_ss(d_tmem, da, db, idesc, accum);
          }
          umma_commit(&empty[stage]);  // frees the stage once these MMAs retire
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        umma_commit(&acc_full[acc]);
      }
    mma_done:;
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kNumEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const int m0 = (t / tiles_n) * kBM;
      const int n0 = (t % tiles_n) * BN;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_phase, args.err, abort_flag))) break;
      tc_fence_after();
      const int m = m0 + row;
      float rs = 1.0f;
      // Raw int32 output (RB_DTYPE_I32) carries no scales.
      if (Cfg::I8 && m < M && args.out_dtype != RB_DTYPE_I32) rs = args.s_row[m];
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld16(tmem_addr(tmem_base, quarter * 32, acc * BN + c), r);
        tmem_wait_ld();
        if (m < M && n0 + c < N) {
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (Cfg::I8) {
              if (args.out_dtype == RB_DTYPE_I32) {
                v[j] = __uint_as_float(r[j]);
              } else {
                const int n = min(n0 + c + j, N - 1);
                // Order matters for bit parity: f32(acc) * (s_row * s_col).
                float y = __fmul_rn(__int2float_rn(static_cast<int32_t>(r[j])),
                                    __fmul_rn(rs, args.s_col[n]));
                if (args.out_scale != 0.0f) {
                  // static_code(y, 1/out_scale) * out_scale (ext.rs:1236-1238, 1356-1360)
                  // Through an integer code like the reference (`as i8`), so a
                  // code of zero is +0.0, never -0.0.
                  const int code = max(-128, min(127, __float2int_rn(__fmul_rn(y, args.out_inv))));
                  y = __fmul_rn(__int2float_rn(code), args.out_scale);
                }
                v[j] = y;
              }
            } else {
              v[j] = __uint_as_float(r[j]);
            }
          }
          const int64_t base = static_cast<int64_t>(m) * args.ldo + n0 + c;
          const int left = N - (n0 + c);
          store_out8(args.out, args.out_dtype, base, v, left >= 8 ? 8 : left);
          if (left > 8) store_out8(args.out, args.out_dtype, base + 8, v + 8, left >= 16 ? 8 : left - 8);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  } else if (Cfg::B_SRC == BSrc::Q8Dequant && warp >= kDqWarp0) {
    // ------------------------------------------------------------ Q8_0 dequant
    // Each 16-byte chunk of the B stage holds 8 f16 weights of one row. Chunk
    // (row, c) lands at row*128 + ((c ^ (row & 7)) * 16) — the 128-B swizzle
    // TMA would have produced — so UMMA reads it with the same descriptor.
    constexpr int kChunks = BN * 8;
    constexpr int kThreads = kNumDqWarps * 32;
    constexpr int kPer = (kChunks + kThreads - 1) / kThreads;
    const int tid = threadIdx.x - kDqWarp0 * 32;
    const int kblocks32 = K / 32;
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      const int n0 = (t % tiles_n) * BN;
      // Prefetch registers for k-block 0.
      uint2 codes[kPer];
      __half sc[kPer];
      auto load_kb = [&](int kb) {
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int i = tid + j * kThreads;
          const int rowi = i >> 3, c = i & 7;
          const int n = n0 + rowi;
          const int k = kb * 64 + c * 8;
          if (i < kChunks && n < N && k < K) {
            codes[j] = __ldg(reinterpret_cast<const uint2*>(args.w_codes +
                                                            static_cast<int64_t>(n) * K + k));
            sc[j] = args.w_scales[static_cast<int64_t>(n) * kblocks32 + (k >> 5)];
          } else {
            codes[j] = make_uint2(0u, 0u);
            sc[j] = __ushort_as_half(0);
          }
        }
      };
      load_kb(0);
      for (int kb = 0; kb < num_kb; ++kb) {
        uint2 cur[kPer];
        __half cur_sc[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) { cur[j] = codes[j]; cur_sc[j] = sc[j]; }
        if (kb + 1 < num_kb) load_kb(kb + 1);
        if (!__all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1, args.err, abort_flag)))
          goto dq_done;
        uint8_t* sb = smem + stage * Cfg::STAGE_BYTES + Cfg::A_BYTES;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int i = tid + j * kThreads;
          if (i < kChunks) {
            const int rowi = i >> 3, c = i & 7;
            const uint4 w = q8_dequant8_f16(cur[j], cur_sc[j]);
            *reinterpret_cast<uint4*>(sb + rowi * 128 + ((c ^ (rowi & 7)) << 4)) = w;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_b[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  dq_done:;
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_after_abort();  // let in-flight TMA / UMMA work retire
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// --------------------------------------------------------------------------
// Host-side launch helpers.

template <class Cfg>
static int launch_gemm(const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmArgs& a,
                       int num_sms, cudaStream_t stream) {
  const int tiles = ((a.M + kBM - 1) / kBM) * ((a.N + Cfg::BN - 1) / Cfg::BN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  static uint64_t configured = 0;  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    if (cudaFuncSetAttribute(gemm_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg::SMEM_BYTES) != cudaSuccess)
      return RB_E_DEVICE;
    configured |= 1ull << (dev & 63);
  }
  gemm_kernel<Cfg><<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(tmA, tmB, a);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

using CfgQ8_256 = GemmCfg<256, 4, false, BSrc::Q8Dequant>;
using CfgQ8_128 = GemmCfg<128, 6, false, BSrc::Q8Dequant>;
using CfgQ8_96 = GemmCfg<96, 6, false, BSrc::Q8Dequant>;
using CfgQ8_64 = GemmCfg<64, 8, false, BSrc::Q8Dequant>;
using CfgI8_256 = GemmCfg<256, 4, true, BSrc::Tma>;
using CfgI8_128 = GemmCfg<128, 6, true, BSrc::Tma>;

// Pick the N tile minimising the makespan of the persistent grid: rounds of
// tiles per SM times the per-tile cost (proportional to BN plus a fixed
// pipeline fill / epilogue overhead expressed in BN units).
static int pick_bn(int M, int N, int num_sms, const int* cands, int ncands) {
  const long tm = (M + kBM - 1) / kBM;
  int best = cands[0];
  long best_cost = -1;
  for (int i = 0; i < ncands; ++i) {
    const int bn = cands[i];
    const long tiles = tm * ((N + bn - 1) / bn);
    const long rounds = (tiles + num_sms - 1) / num_sms;
    const long cost = rounds * (bn + 32);
    if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = bn; }
  }
  return best;
}

int launch_q8_gemm(const CUtensorMap& tmA, const GemmLaunch& L, cudaStream_t stream) {
  GemmArgs a{};
  a.M = L.M; a.N = L.N; a.K = L.K;
  a.w_codes = L.w_codes; a.w_scales = reinterpret_cast<const __half*>(L.w_scales);
  a.out = L.out; a.ldo = L.ldo; a.out_dtype = L.out_dtype; a.err = L.err;
  static const int cands[] = {256, 128, 96, 64};
  int bn = L.force_bn ? L.force_bn : pick_bn(L.M, L.N, L.num_sms, cands, 4);
  CUtensorMap dummy = tmA;
  switch (bn) {
    case 256: return launch_gemm<CfgQ8_256>(tmA, dummy, a, L.num_sms, stream);
    case 128: return launch_gemm<CfgQ8_128>(tmA, dummy, a, L.num_sms, stream);
    case 96: return launch_gemm<CfgQ8_96>(tmA, dummy, a, L.num_sms, stream);
    case 64: return launch_gemm<CfgQ8_64>(tmA, dummy, a, L.num_sms, stream);
    default: return RB_E_SHAPE;
  }
}

int launch_w8a8_gemm(const CUtensorMap& tmA, const CUtensorMap& tmB256,
                     const CUtensorMap& tmB128, const GemmLaunch& L, cudaStream_t stream) {
  GemmArgs a{};
  a.M = L.M; a.N = L.N; a.K = L.K;
  a.s_row = L.s_row; a.s_col = L.s_col;
  a.out_scale = L.out_scale;
  a.out_inv = L.out_scale != 0.0f ? 1.0f / L.out_scale : 0.0f;
  a.out = L.out; a.ldo = L.ldo; a.out_dtype = L.out_dtype; a.err = L.err;
  static const int cands[] = {256, 128};
  int bn = L.force_bn ? L.force_bn : pick_bn(L.M, L.N, L.num_sms, cands, 2);
  switch (bn) {
    case 256: return launch_gemm<CfgI8_256>(tmA, tmB256, a, L.num_sms, stream);
    case 128: return launch_gemm<CfgI8_128>(tmA, tmB128, a, L.num_sms, stream);
    default: return RB_E_SHAPE;
  }
}

// --------------------------------------------------------------------------
// Standalone dequantisation kernels (debug / parity surface of the codec).

// f32 = f32(d) * f32(q), exact (gguf.rs:197-215).
__global__ void q8_dequant_f32_kernel(const int8_t* codes, const __half* scales, int N, int K,
                                      float* out) {
  const int64_t total = static_cast<int64_t>(N) * K;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / K, k = i % K;
    const float d = __half2float(scales[n * (K / 32) + k / 32]);
    out[i] = __fmul_rn(d, static_cast<float>(codes[i]));
  }
}

// f16 = RNE(d * q): the exact values the GEMM's producer warps stage.
__global__ void q8_dequant_f16_kernel(const int8_t* codes, const __half* scales, int N, int K,
                                      __half* out) {
  const int64_t total8 = static_cast<int64_t>(N) * K / 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const int64_t n = e / K, k = e % K;
    const uint2 c = *reinterpret_cast<const uint2*>(codes + e);
    const uint4 w = q8_dequant8_f16(c, scales[n * (K / 32) + k / 32]);
    *reinterpret_cast<uint4*>(out + e) = w;
  }
}

int launch_q8_dequant(const int8_t* codes, const void* scales, int N, int K, void* out,
                      bool f16_out, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(N) * K;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (f16_out)
    q8_dequant_f16_kernel<<<static_cast<int>(blocks), threads, 0, stream>>>(
        codes, reinterpret_cast<const __half*>(scales), N, K, reinterpret_cast<__half*>(out));
  else
    q8_dequant_f32_kernel<<<static_cast<int>(blocks), threads, 0, stream>>>(
        codes, reinterpret_cast<const __half*>(scales), N, K, reinterpret_cast<float*>(out));
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

}  // namespace rb
