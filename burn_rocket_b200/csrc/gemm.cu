// gemm.cu — persistent tcgen05 GEMMs for the two resident-weight matmul kinds
// burn-rocket offloads:
//
//   * Q8_0:  C[M,N] = A[M,K] (f16) · deq(W)[N,K]^T with deq(W) = f16(d · q).
//            The int8 codes and the f16 block scales (one per 32 K values) are
//            staged into shared memory by TMA and dequantised there, by
//            producer warps, into the 128-byte-swizzled K-major layout that
//            kind::f16 UMMA reads; accumulation is f32 in TMEM. (Reference
//            semantics: the NPU route packs dequantised Q8_0 as fp16,
//            crates/burn-rocket/src/ext.rs:1437-1499; the codec is
//            src/util/gguf.rs:197-215.)
//   * W8A8:  acc[M,N] = Aq[M,K] (s8) · Wq[N,K]^T (s8) on kind::i8 UMMA with an
//            s32 TMEM accumulator; epilogue y = f32(acc) · (s_row[m] · s_col[n])
//            in exactly that order (ext.rs:1350-1363).
//
// Q8_0 weight planes in HBM (written at pack time):
//   codes  int8 [N, K] row-major
//   scales f16  [K/32, pitch], pitch = round_up(N, 8) (k-block-major: one TMA
//                           box carries the two scales of a 64-wide K stage
//                           for BN weight rows)
//
// Warp roles (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer (A and B, or A + codes + scales)
//   warp 1      UMMA issuer (one elected lane) and TMEM owner
//   warps 2..5  epilogue: TMEM -> registers -> swizzled smem -> TMA store
//   warps 6..13 Q8_0 only: dequantise staged codes into the f16 B ring
// The accumulator is double-buffered in TMEM so the epilogue of tile i
// overlaps the main loop of tile i+1.
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "sm100.cuh"
#include "kernels.h"

namespace rb {

constexpr int kEpiWarp0 = 2;      // first epilogue warp
constexpr int kNumEpiWarps = 4;
constexpr int kDqWarp0 = 6;       // first dequant warp (Q8_0 only)
constexpr int kNumDqWarps = 8;
constexpr int kEpiBufBytes = 4096;  // 32 rows x 128 B, one per warp and buffer

enum class BSrc { Tma, Q8Dequant };

constexpr int round1k(int x) { return (x + 1023) & ~1023; }

template <int BN_, int LSTAGES_, bool I8_, int BSTAGES_ = 2, int MH_ = 1>
struct GemmCfg {
  static constexpr int BN = BN_;
  // 128-row M halves per tile: MH = 2 issues two M=128 UMMAs per K step that
  // share one (dequantised) B tile, halving the dequant work per FLOP.
  static constexpr int MH = MH_;
  static constexpr int BM = 128 * MH;
  static constexpr int LSTAGES = LSTAGES_;          // TMA load ring depth
  static constexpr bool I8 = I8_;
  static constexpr bool Q8 = !I8;
  static constexpr int BSTAGES = BSTAGES_;          // dequantised B ring (Q8_0)
  static constexpr int ELEM = I8 ? 1 : 2;
  static constexpr int BK = 128 / ELEM;             // K elements per stage (one 128-B atom)
  static constexpr int UMMA_K = I8 ? 32 : 16;
  static constexpr int KSTEPS = BK / UMMA_K;        // 4
  static constexpr int A_BYTES = BM * 128;          // 16 KB per M half
  static constexpr int B_BYTES = BN * 128;          // one B tile (f16 or s8)
  static constexpr int CODE_BYTES = Q8 ? BN * 64 : 0;
  static constexpr int SC_BYTES = Q8 ? 2 * BN * 2 : 0;
  static constexpr int LOAD_TX = Q8 ? (A_BYTES + CODE_BYTES + SC_BYTES) : (A_BYTES + B_BYTES);
  static constexpr int LSTAGE = round1k(LOAD_TX);
  static constexpr int BRING_OFF = LSTAGES * LSTAGE;
  static constexpr int BRING = Q8 ? BSTAGES * B_BYTES : 0;
  static constexpr int EPI_OFF = BRING_OFF + BRING;
  static constexpr int EPI_BYTES = kNumEpiWarps * 2 * kEpiBufBytes;
  static constexpr int BAR_OFF = EPI_OFF + EPI_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 384 + 1024;
  static constexpr int NUM_WARPS = Q8 ? (kDqWarp0 + kNumDqWarps) : 6;
  static constexpr int THREADS = NUM_WARPS * 32;
  static constexpr int ACC_COLS = MH * BN;          // one accumulator (all M halves)
  static constexpr uint32_t TMEM_COLS = (2 * ACC_COLS <= 32) ? 32 : (2 * ACC_COLS <= 64) ? 64
                                        : (2 * ACC_COLS <= 128) ? 128 : (2 * ACC_COLS <= 256) ? 256 : 512;
  static_assert(2 * ACC_COLS <= 512, "two accumulators must fit in TMEM");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N constraint for M=128");
  static_assert(B_BYTES % 1024 == 0, "B tiles must keep 1024-byte alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

struct GemmArgs {
  int M, N, K;
  const float* s_row;  // W8A8 [M]
  const float* s_col;  // W8A8 [N]
  void* out;           // [M, ldo]
  int ldo;
  int out_dtype;       // RB_DTYPE_* (RB_DTYPE_I32: raw int8-GEMM accumulators)
  float out_scale;     // W8A8: calibrated output grid (0 = unrounded)
  float out_inv;       // 1 / out_scale in f32
  int tma_store;       // epilogue through smem + TMA store (else direct stores)
  uint32_t* err;
};

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

// Epilogue modes of the TMA-store path, fixed per launch: raw 4-byte
// accumulators (f32 for Q8_0, s32 for RB_DTYPE_I32), f16 / bf16 casts, and the
// W8A8 scaled forms (kEpiS8*; Q = onto the calibrated output grid).
enum : int {
  kEpiRaw4 = 0, kEpiF16, kEpiBF16,
  kEpiS8F32, kEpiS8F16, kEpiS8BF16, kEpiS8F32Q, kEpiS8F16Q, kEpiS8BF16Q
};

__host__ __device__ __forceinline__ int epi_mode(bool i8, int out_dtype, float out_scale) {
  const int cast = out_dtype == RB_DTYPE_F16 ? 1 : out_dtype == RB_DTYPE_BF16 ? 2 : 0;
  if (!i8 || out_dtype == RB_DTYPE_I32) return out_dtype == RB_DTYPE_I32 ? kEpiRaw4 : cast;
  return kEpiS8F32 + cast + (out_scale != 0.0f ? 3 : 0);
}

// One 32-row x 128-byte chunk of the output tile, written into the
// 128-byte-swizzled staging row `b` of this lane: columns [0, CW) of the chunk
// from accumulator registers ra (0..31) and rb (32..63, 2-byte outputs only).
// SCALE applies the W8A8 epilogue f32(acc) * (rs * s_col[n]) — in that order,
// for bit parity with ext.rs:1350-1363 — with the chunk's column scales read
// as float4 vectors up front (scp = s_col + first column; nvalid columns are
// in range, the rest clamp to the last valid one and are clipped by the TMA
// store). OUT is the output element size in bytes' role: 4 (f32 / raw), 1 (f16),
// 2 (bf16). QGRID rounds onto the static output grid (ext.rs:1236-1238).
template <bool SCALE, int OUT, bool QGRID>
__device__ __forceinline__ void epi_chunk(uint8_t* b, int lane, const uint32_t (&ra)[32],
                                          const uint32_t (&rb)[32], float rs, const float* scp,
                                          int nvalid, const EpiParams& ep) {
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
    if constexpr (!SCALE) {
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
    *reinterpret_cast<uint4*>(b + ((j ^ (lane & 7)) << 4)) = o;
  }
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmC,
            GemmArgs args) {
  constexpr int BN = Cfg::BN;
  constexpr int LSTAGES = Cfg::LSTAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t* load_full = bars;                       // [LSTAGES] TMA bytes
  uint64_t* load_empty = bars + LSTAGES;            // [LSTAGES] UMMA (+ dequant warps)
  uint64_t* b_full = bars + 2 * LSTAGES;            // [BSTAGES] dequant warps (Q8_0)
  uint64_t* b_empty = b_full + Cfg::BSTAGES;        // [BSTAGES] UMMA (Q8_0)
  uint64_t* acc_full = b_empty + Cfg::BSTAGES;      // [2]
  uint64_t* acc_empty = acc_full + 2;               // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = args.M, N = args.N, K = args.K;
  const int tiles_n = (N + BN - 1) / BN;
  const int tiles_m = (M + Cfg::BM - 1) / Cfg::BM;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + Cfg::BK - 1) / Cfg::BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < LSTAGES; ++s) {
      mbar_init(&load_full[s], 1);
      mbar_init(&load_empty[s], Cfg::Q8 ? 1 + kNumDqWarps : 1);
    }
    for (int i = 0; i < Cfg::BSTAGES; ++i) {
      mbar_init(&b_full[i], kNumDqWarps);
      mbar_init(&b_empty[i], 1);
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
    tma_prefetch_desc(&tmB);
    if (Cfg::Q8) tma_prefetch_desc(&tmS);
    if (args.tma_store) tma_prefetch_desc(&tmC);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one_sync()) {
      int ls = 0;
      uint32_t lph = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        const int m0 = (t / tiles_n) * Cfg::BM;
        const int n0 = (t % tiles_n) * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&load_empty[ls], lph ^ 1, args.err, abort_flag)) goto producer_done;
          uint8_t* st = smem + ls * Cfg::LSTAGE;
          mbar_arrive_expect_tx(&load_full[ls], Cfg::LOAD_TX);
          tma_load_2d(st, &tmA, &load_full[ls], kb * Cfg::BK, m0);
          if (Cfg::I8) {
            tma_load_2d(st + Cfg::A_BYTES, &tmB, &load_full[ls], kb * Cfg::BK, n0);
          } else {
            tma_load_2d(st + Cfg::A_BYTES, &tmB, &load_full[ls], kb * 64, n0);
            tma_load_2d(st + Cfg::A_BYTES + Cfg::CODE_BYTES, &tmS, &load_full[ls], n0, kb * 2);
          }
          if (++ls == LSTAGES) { ls = 0; lph ^= 1; }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t idesc =
          Cfg::I8 ? idesc_i8(128, BN) : idesc_f16(128, BN, false, false, false);
      int ls = 0, bs = 0;
      uint32_t lph = 0, bph = 0;
      int local = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, args.err, abort_flag)) goto mma_done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * Cfg::ACC_COLS;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&load_full[ls], lph, args.err, abort_flag)) goto mma_done;
          if (Cfg::Q8) {
            if (!mbar_wait(&b_full[bs], bph, args.err, abort_flag)) goto mma_done;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + ls * Cfg::LSTAGE);
          const uint32_t b_addr = Cfg::Q8 ? smem_u32(smem + Cfg::BRING_OFF + bs * Cfg::B_BYTES)
                                          : a_addr + Cfg::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < Cfg::KSTEPS; ++ks) {
            const uint64_t db = desc_kmajor_sw128(b_addr + ks * 32);
            const uint32_t accum = (kb > 0 || ks > 0) ? 1u : 0u;
#pragma unroll
            for (int h = 0; h < Cfg::MH; ++h) {  // M halves share the B tile
              const uint64_t da = desc_kmajor_sw128(a_addr + h * 16384 + ks * 32);
              if (Cfg::I8) umma_i8_ss(d_tmem + h * BN, da, db, idesc, accum);
              else umma_f16_ss(d_tmem + h * BN, da, db, idesc, accum);
            }
          }
          umma_commit(&load_empty[ls]);  // frees the load stage once these MMAs retire
          if (++ls == LSTAGES) { ls = 0; lph ^= 1; }
          if (Cfg::Q8) {
            umma_commit(&b_empty[bs]);
            if (++bs == Cfg::BSTAGES) { bs = 0; bph ^= 1; }
          }
        }
        umma_commit(&acc_full[acc]);
      }
    mma_done:;
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kNumEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const EpiParams ep{args.s_col, args.out_dtype, args.out_scale, args.out_inv};
    uint8_t* ebuf = smem + Cfg::EPI_OFF + (warp - kEpiWarp0) * 2 * kEpiBufBytes;
    const int out_bytes = (args.out_dtype == RB_DTYPE_F16 || args.out_dtype == RB_DTYPE_BF16) ? 2 : 4;
    const int CW = 128 / out_bytes;  // columns per 128-byte store row
    const int mode = epi_mode(Cfg::I8, args.out_dtype, args.out_scale);
    int buf = 0;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const int n0 = (t % tiles_n) * BN;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!warp_wait(&acc_full[acc], acc_phase, args.err, abort_flag)) break;
      tc_fence_after();
      for (int h = 0; h < Cfg::MH; ++h) {
      const int m0 = (t / tiles_n) * Cfg::BM + h * 128;
      const uint32_t acc_col = acc * Cfg::ACC_COLS + h * BN;
      const int m = m0 + row;
      float rs = 1.0f;
      // Raw int32 output (RB_DTYPE_I32) carries no scales.
      if (Cfg::I8 && m < M && args.out_dtype != RB_DTYPE_I32) rs = args.s_row[m];
      const bool rows_live = m0 + quarter * 32 < M;  // warp-uniform
      if (args.tma_store) {
        if (rows_live) {
          for (int c0 = 0; c0 < BN && n0 + c0 < N; c0 += CW) {
            uint32_t ra[32], rb[32];  // columns c0..c0+31 and (2-byte outputs) c0+32..c0+63
            tmem_ld32(tmem_addr(tmem_base, quarter * 32, acc_col + c0), ra);
            if (CW == 64) tmem_ld32(tmem_addr(tmem_base, quarter * 32, acc_col + c0 + 32), rb);
            tmem_wait_ld();
            // The buffer about to be written must have been read by its
            // previous TMA store (at most one store of this warp in flight).
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
            uint8_t* b = ebuf + buf * kEpiBufBytes + lane * 128;
            const float* scp = Cfg::I8 ? ep.s_col + n0 + c0 : nullptr;
            const int nvalid = N - (n0 + c0);
            switch (mode) {
              case kEpiRaw4: epi_chunk<false, 4, false>(b, lane, ra, rb, rs, scp, nvalid, ep); break;
              case kEpiF16: epi_chunk<false, 1, false>(b, lane, ra, rb, rs, scp, nvalid, ep); break;
              case kEpiBF16: epi_chunk<false, 2, false>(b, lane, ra, rb, rs, scp, nvalid, ep); break;
              default:
                if constexpr (Cfg::I8) {
                  switch (mode) {
                    case kEpiS8F32: epi_chunk<true, 4, false>(b, lane, ra, rb, rs, scp, nvalid, ep); break;
                    case kEpiS8F16: epi_chunk<true, 1, false>(b, lane, ra, rb, rs, scp, nvalid, ep); break;
                    case kEpiS8BF16: epi_chunk<true, 2, false>(b, lane, ra, rb, rs, scp, nvalid, ep); break;
                    case kEpiS8F32Q: epi_chunk<true, 4, true>(b, lane, ra, rb, rs, scp, nvalid, ep); break;
                    case kEpiS8F16Q: epi_chunk<true, 1, true>(b, lane, ra, rb, rs, scp, nvalid, ep); break;
                    default: epi_chunk<true, 2, true>(b, lane, ra, rb, rs, scp, nvalid, ep); break;
                  }
                }
                break;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmC, ebuf + buf * kEpiBufBytes, n0 + c0, m0 + quarter * 32);
              bulk_commit();
            }
            buf ^= 1;
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          uint32_t r[16];
          tmem_ld16(tmem_addr(tmem_base, quarter * 32, acc_col + c), r);
          tmem_wait_ld();
          if (m < M && n0 + c < N) {
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = epi_value<Cfg::I8>(ep, r[j], rs, min(n0 + c + j, N - 1));
            const int64_t base = static_cast<int64_t>(m) * args.ldo + n0 + c;
            store_out16(args.out, ep.out_dtype, base, v, N - (n0 + c));
          }
        }
      }
      }  // M halves
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
    if (args.tma_store && lane == 0) bulk_wait_all<0>();  // stores complete before exit
  } else if (Cfg::Q8 && warp >= kDqWarp0) {
    // ------------------------------------------------------------ Q8_0 dequant
    // Chunk (row, c) — 8 codes of one weight row — is read from the staged
    // codes at row*64 + c*8 and written as 8 f16 at row*128 + ((c ^ (row&7))*16):
    // the 128-byte swizzle TMA would produce, read by UMMA with the same
    // descriptor as any other K-major operand.
    constexpr int kChunks = BN * 8;
    constexpr int kThreads = kNumDqWarps * 32;
    constexpr int kPer = (kChunks + kThreads - 1) / kThreads;
    const int tid = threadIdx.x - kDqWarp0 * 32;
    int ls = 0, bs = 0;
    uint32_t lph = 0, bph = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!warp_wait(&load_full[ls], lph, args.err, abort_flag)) goto dq_done;
        if (!warp_wait(&b_empty[bs], bph ^ 1, args.err, abort_flag)) goto dq_done;
        const uint8_t* codes = smem + ls * Cfg::LSTAGE + Cfg::A_BYTES;
        const __half* sc = reinterpret_cast<const __half*>(codes + Cfg::CODE_BYTES);
        uint8_t* sb = smem + Cfg::BRING_OFF + bs * Cfg::B_BYTES;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int i = tid + j * kThreads;
          if (kChunks % kThreads == 0 || i < kChunks) {
            const int rowi = i >> 3, c = i & 7;
            const uint2 q = *reinterpret_cast<const uint2*>(codes + rowi * 64 + c * 8);
            const __half d = sc[(c >> 2) * BN + rowi];
            *reinterpret_cast<uint4*>(sb + rowi * 128 + ((c ^ (rowi & 7)) << 4)) =
                q8_dequant8_f16(q, d);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&b_full[bs]);
          mbar_arrive(&load_empty[ls]);  // staged codes consumed
        }
        if (++ls == LSTAGES) { ls = 0; lph ^= 1; }
        if (++bs == Cfg::BSTAGES) { bs = 0; bph ^= 1; }
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
// Host-side launch.

// Q8_0: (BN, load-ring depth, dequantised-B-ring depth) sized to the smem budget.
using CfgQ8_256 = GemmCfg<256, 3, false, 2>;
using CfgQ8_128 = GemmCfg<128, 4, false, 4>;
using CfgQ8_96 = GemmCfg<96, 4, false, 6>;
using CfgQ8_64 = GemmCfg<64, 6, false, 6>;
using CfgQ8_128x2 = GemmCfg<128, 3, false, 3, 2>;  // 256-row M tile
using CfgI8_256 = GemmCfg<256, 4, true>;
using CfgI8_128 = GemmCfg<128, 6, true>;

template <class Cfg>
static int launch_cfg(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmS,
                      const CUtensorMap* tmC, const GemmArgs& a, int num_sms,
                      cudaStream_t stream) {
  const int tiles = ((a.M + Cfg::BM - 1) / Cfg::BM) * ((a.N + Cfg::BN - 1) / Cfg::BN);
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
  GemmArgs args = a;
  const int out_bytes = (a.out_dtype == RB_DTYPE_F16 || a.out_dtype == RB_DTYPE_BF16) ? 2 : 4;
  // The TMA-store epilogue writes whole 128-byte rows of the N tile.
  args.tma_store = tmC != nullptr && (Cfg::BN % (128 / out_bytes)) == 0;
  gemm_kernel<Cfg><<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(tmA, tmB, tmS,
                                                                     tmC ? *tmC : tmA, args);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

// Tile shape (BN, M halves) minimising the makespan of the persistent grid:
// rounds of tiles per SM times the per-tile cost. A tile's cost is its MMA
// work (MH * BN columns of 128 rows) scaled by how well the shape feeds the
// tensor core — a Q8_0 tile with one M half spends twice the dequant work per
// FLOP — plus a fixed pipeline fill / epilogue overhead.
void gemm_pick(bool i8, int M, int N, int num_sms, int* bn_out, int* mh_out) {
  struct Shape { int bn, mh; double eff; };
  static const Shape q8c[] = {{256, 1, 1.4}, {128, 1, 1.4}, {96, 1, 1.4}, {64, 1, 1.4}, {128, 2, 1.0}};
  static const Shape i8c[] = {{256, 1, 1.0}, {128, 1, 1.0}};
  const Shape* c = i8 ? i8c : q8c;
  const int nc = i8 ? 2 : 5;
  double best_cost = -1.0;
  for (int i = 0; i < nc; ++i) {
    const long tiles = ((M + 128L * c[i].mh - 1) / (128L * c[i].mh)) * ((N + c[i].bn - 1) / c[i].bn);
    const long rounds = (tiles + num_sms - 1) / num_sms;
    const double cost = rounds * (c[i].mh * c[i].bn * c[i].eff + 32.0);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      *bn_out = c[i].bn;
      *mh_out = c[i].mh;
    }
  }
}

static GemmArgs make_args(const GemmLaunch& L) {
  GemmArgs a{};
  a.M = L.M; a.N = L.N; a.K = L.K;
  a.s_row = L.s_row; a.s_col = L.s_col;
  a.out = L.out; a.ldo = L.ldo; a.out_dtype = L.out_dtype;
  a.out_scale = L.out_scale;
  a.out_inv = L.out_scale != 0.0f ? 1.0f / L.out_scale : 0.0f;
  a.err = L.err;
  return a;
}

int launch_q8_gemm(const GemmLaunch& L, int bn, int mh, const CUtensorMap& tmA,
                   const CUtensorMap& tmCodes, const CUtensorMap& tmScales, const CUtensorMap* tmC,
                   cudaStream_t stream) {
  const GemmArgs a = make_args(L);
  if (mh == 2) {
    if (bn != 128) return RB_E_SHAPE;
    return launch_cfg<CfgQ8_128x2>(tmA, tmCodes, tmScales, tmC, a, L.num_sms, stream);
  }
  switch (bn) {
    case 256: return launch_cfg<CfgQ8_256>(tmA, tmCodes, tmScales, tmC, a, L.num_sms, stream);
    case 128: return launch_cfg<CfgQ8_128>(tmA, tmCodes, tmScales, tmC, a, L.num_sms, stream);
    case 96: return launch_cfg<CfgQ8_96>(tmA, tmCodes, tmScales, tmC, a, L.num_sms, stream);
    case 64: return launch_cfg<CfgQ8_64>(tmA, tmCodes, tmScales, tmC, a, L.num_sms, stream);
    default: return RB_E_SHAPE;
  }
}

int launch_w8a8_gemm(const GemmLaunch& L, int bn, const CUtensorMap& tmA, const CUtensorMap& tmB,
                     const CUtensorMap* tmC, cudaStream_t stream) {
  const GemmArgs a = make_args(L);
  switch (bn) {
    case 256: return launch_cfg<CfgI8_256>(tmA, tmB, tmA, tmC, a, L.num_sms, stream);
    case 128: return launch_cfg<CfgI8_128>(tmA, tmB, tmA, tmC, a, L.num_sms, stream);
    default: return RB_E_SHAPE;
  }
}

// --------------------------------------------------------------------------
// Standalone dequantisation kernels (the codec's parity surface).

// f32 = f32(d) * f32(q), exact (gguf.rs:197-215). scales are [K/32, N].
__global__ void q8_dequant_f32_kernel(const int8_t* codes, const __half* scales, int N, int K,
                                      int pitch, float* out) {
  const int64_t total = static_cast<int64_t>(N) * K;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / K, k = i % K;
    const float d = __half2float(scales[(k / 32) * pitch + n]);
    out[i] = __fmul_rn(d, static_cast<float>(codes[i]));
  }
}

// f16 = RNE(d * q): the exact values the GEMM's producer warps stage.
__global__ void q8_dequant_f16_kernel(const int8_t* codes, const __half* scales, int N, int K,
                                      int pitch, __half* out) {
  const int64_t total8 = static_cast<int64_t>(N) * K / 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const int64_t n = e / K, k = e % K;
    const uint2 c = *reinterpret_cast<const uint2*>(codes + e);
    const uint4 w = q8_dequant8_f16(c, scales[(k / 32) * pitch + n]);
    *reinterpret_cast<uint4*>(out + e) = w;
  }
}

int launch_q8_dequant(const int8_t* codes, const void* scales, int N, int K, int pitch, void* out,
                      bool f16_out, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(N) * K;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (f16_out)
    q8_dequant_f16_kernel<<<static_cast<int>(blocks), threads, 0, stream>>>(
        codes, reinterpret_cast<const __half*>(scales), N, K, pitch, reinterpret_cast<__half*>(out));
  else
    q8_dequant_f32_kernel<<<static_cast<int>(blocks), threads, 0, stream>>>(
        codes, reinterpret_cast<const __half*>(scales), N, K, pitch, reinterpret_cast<float*>(out));
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

}  // namespace rb
