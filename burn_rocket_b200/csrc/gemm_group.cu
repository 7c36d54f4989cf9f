// gemm_group.cu — group-wise int8 GEMM with the group promotion inside the
// kernel (matmul_i8 / matmul_gw: crates/burn-rocket/src/ext.rs:1505-1554,
// crates/rocket-npu/src/matmul/int8.rs:641-672):
//
//   C[m, n] = sum over the K groups g, in order, of
//             f32(a_s[m, g] * b_s[n, g]) * f32(P_g[m, n]),
//   P_g = A_g · B_g^T, the exact int32 product of the group's K slice of the
//   int8 activation codes A and weight codes B.
//
// One persistent CTA per SM walks 128 x 128 output tiles:
//   warp 0      TMA producer: 128 x 128 int8 stages of A and B
//   warp 1      UMMA issuer and TMEM owner: kind::i8 UMMAs (K = 32 each)
//               write each group's int32 partial into the next buffer of a
//               ring of three 128-column TMEM buffers (the group's first K
//               step starts the buffer at zero) and commit it at the group's
//               last K step
//   warps 2..9  fold: as soon as a group's partial lands, each warp loads its
//               32 rows x 64 columns of it, releases the buffer, and adds
//               f32(a_s * b_s) * f32(partial) into f32 registers — the
//               reference's order, every operation individually rounded (the
//               multiplies two columns per packed f32x2 instruction, each
//               lane IEEE-rounded on its own; the accumulating adds scalar,
//               never contracted with a multiply), so the result is
//               bit-identical. The MMA of the next groups runs
//               while the fold works. At the end of the tile the f32 sums go
//               to a fourth TMEM buffer and leave through the shared GEMM
//               epilogue (swizzled staging + TMA store; f16 / bf16 casts).
// No partial ever goes through global memory: per call there are two
// launches, the activation group quantiser and this kernel.
//
// f32(partial): |P_g| <= 127 * 127 * G, below 2^22 for G <= 256, where the
// int32 -> f32 conversion is exact and is done on the FP32 pipe (adding the
// integer to the bits of 1.5 * 2^23 and subtracting 1.5 * 2^23); larger
// groups use the conversion instruction (rounding to nearest even either way,
// as the reference's `as f32`).
#include "gemm_common.cuh"

namespace rb {

namespace {
constexpr int kGBN = 128;                    // tile columns (UMMA N)
constexpr int kGBK = 128;                    // K (int8) per stage: one 128-byte swizzle atom
constexpr int kGStages = 5;
constexpr int kGParts = 3;                   // partial buffers in TMEM (columns 0..383)
constexpr int kGOutCol = kGParts * kGBN;     // f32 result buffer (columns 384..511)
constexpr int kGEpiWarps = 8;                // two per TMEM lane quarter (column halves)
constexpr int kGHalf = kGBN / 2;             // columns per fold warp
constexpr int kGStageBytes = 2 * 128 * 128;  // A + B
constexpr int kGEpiOff = kGStages * kGStageBytes;
constexpr int kGBarOff = kGEpiOff + kGEpiWarps * kEpiBufBytes;
constexpr int kGSmem = kGBarOff + 256 + 1024;
constexpr int kGThreads = (kEpiWarp0 + kGEpiWarps) * 32;
static_assert(kGSmem <= 232448, "shared memory budget");
}  // namespace

struct GroupArgs {
  int M, N, K, G;
  const float* a_s;   // activation group scales [M, K/G]
  const float* b_st;  // weight group scales, group-major [K/G, ldb] (zero past N)
  int ldb;            // >= tiles_n * 128
  void* out;
  int ldo;
  int out_dtype;
  int epi_path;
  uint32_t* err;
};

// (Packed f32x2 helpers: sm100.cuh. The accumulating adds below stay scalar
// add.rn, which is never contracted with a multiply into a single rounding.)

// f32 of two int32 partials. SMALL (|p| < 2^22): 1.5 * 2^23 + p is exact with
// ulp 1, so adding the integer to the bits of 1.5 * 2^23 and subtracting
// 1.5 * 2^23 is the exact conversion; otherwise the conversion instruction.
template <bool SMALL>
__device__ __forceinline__ uint64_t group_part_f32x2(uint32_t p0, uint32_t p1) {
  if constexpr (SMALL) {
    const uint64_t m = f2_pack(__int_as_float(static_cast<int>(p0) + 0x4B400000),
                               __int_as_float(static_cast<int>(p1) + 0x4B400000));
    return f2_add(m, f2_pack(-12582912.0f, -12582912.0f));  // exact: no rounding involved
  } else {
    return f2_pack(__int2float_rn(static_cast<int>(p0)), __int2float_rn(static_cast<int>(p1)));
  }
}

template <bool SMALL>
__global__ void __launch_bounds__(kGThreads, 1)
gemm_i8g_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, GroupArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kGBarOff);
  uint64_t* load_full = bars;                    // [kGStages] TMA bytes
  uint64_t* load_empty = load_full + kGStages;   // [kGStages] UMMA commit
  uint64_t* part_full = load_empty + kGStages;   // [kGParts] UMMA commit (group's partial complete)
  uint64_t* part_empty = part_full + kGParts;    // [kGParts] fold warps have loaded it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(part_empty + kGParts);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = args.M, N = args.N, K = args.K, G = args.G;
  const int tiles_n = (N + kGBN - 1) / kGBN;
  const int num_tiles = ((M + 127) / 128) * tiles_n;
  const int num_kb = (K + kGBK - 1) / kGBK;
  const int ng = K / G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&load_full[s], 1);
      mbar_init(&load_empty[s], 1);
    }
    for (int i = 0; i < kGParts; ++i) {
      mbar_init(&part_full[i], 1);
      mbar_init(&part_empty[i], kGEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (args.epi_path == kEpiPathTma) tma_prefetch_desc(&tmC);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // the activation codes and group scales come from the quantiser

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one_sync()) {
      int ls = 0;
      uint32_t lph = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        const int m0 = (t / tiles_n) * 128, n0 = (t % tiles_n) * kGBN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&load_empty[ls], lph ^ 1, args.err, abort_flag)) goto producer_done;
          uint8_t* st = smem + ls * kGStageBytes;
          mbar_arrive_expect_tx(&load_full[ls], kGStageBytes);
          tma_load_2d(st, &tmA, &load_full[ls], kb * kGBK, m0);
          tma_load_2d(st + 128 * 128, &tmB, &load_full[ls], kb * kGBK, n0);
          if (++ls == kGStages) { ls = 0; lph ^= 1; }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t idesc = idesc_i8(128, kGBN);
      int ls = 0;
      uint32_t lph = 0;
      int q = 0;  // groups issued so far (partial ring position)
      uint32_t d_tmem = tmem_base;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&load_full[ls], lph, args.err, abort_flag)) goto mma_done;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + ls * kGStageBytes);
          const uint32_t b_addr = a_addr + 128 * 128;
#pragma unroll
          for (int ks = 0; ks < kGBK / 32; ++ks) {
            const int k = kb * kGBK + ks * 32;
            if (k >= K) break;
            const int kin = k % G;
            if (kin == 0) {  // a new group: its partial buffer must have been drained
              const int pb = q % kGParts;
              if (!mbar_wait(&part_empty[pb], ((q / kGParts) & 1) ^ 1, args.err, abort_flag)) goto mma_done;
              tc_fence_after();
              d_tmem = tmem_base + pb * kGBN;
            }
            umma_i8_ss(d_tmem, desc_kmajor_sw128(a_addr + ks * 32), desc_kmajor_sw128(b_addr + ks * 32), idesc,
                       kin != 0 ? 1u : 0u);
            if (kin + 32 == G) {  // the group's last K step
              umma_commit(&part_full[q % kGParts]);
              ++q;
            }
          }
          umma_commit(&load_empty[ls]);  // frees the stage once these MMAs retire
          if (++ls == kGStages) { ls = 0; lph ^= 1; }
        }
      }
    mma_done:;
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kGEpiWarps) {
    // ------------------------------------------------------------ group fold + epilogue
    const int quarter = warp & 3;                     // TMEM lane quarter this warp may access
    const int cbeg = ((warp - kEpiWarp0) >> 2) * kGHalf;
    const EpiParams ep{nullptr, args.out_dtype, 0.0f, 0.0f};
    const int mode = epi_mode(false, args.out_dtype, 0.0f);
    uint8_t* ebuf = smem + kGEpiOff + (warp - kEpiWarp0) * kEpiBufBytes;
    int buf = 0;
    int q = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      const int m0 = (t / tiles_n) * 128, n0 = (t % tiles_n) * kGBN;
      const int m = min(m0 + quarter * 32 + lane, M - 1);
      const float* asr = args.a_s + static_cast<int64_t>(m) * ng;
      float acc[kGHalf];
#pragma unroll
      for (int c = 0; c < kGHalf; ++c) acc[c] = 0.0f;
      for (int g = 0; g < ng; ++g, ++q) {
        const int pb = q % kGParts;
        if (!warp_wait(&part_full[pb], (q / kGParts) & 1, args.err, abort_flag)) goto fold_done;
        tc_fence_after();
        uint32_t p[kGHalf];
        const uint32_t taddr = tmem_addr(tmem_base, quarter * 32, pb * kGBN + cbeg);
        tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&p[0]));
        tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&p[32]));
        const float a = __ldg(asr + g);  // scale loads in flight with the TMEM loads
        const float4* bs = reinterpret_cast<const float4*>(args.b_st + static_cast<int64_t>(g) * args.ldb + n0 +
                                                           cbeg);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&part_empty[pb]);  // the MMA may refill this buffer
        const uint64_t aa = f2_pack(a, a);
#pragma unroll
        for (int c4 = 0; c4 < kGHalf / 4; ++c4) {
          const float4 b4 = __ldg(bs + c4);
          // f32(a_s * b_s), then f32(that * f32(partial)), two columns per instruction
          const uint64_t t01 = f2_mul(f2_mul(aa, f2_pack(b4.x, b4.y)),
                                      group_part_f32x2<SMALL>(p[4 * c4], p[4 * c4 + 1]));
          const uint64_t t23 = f2_mul(f2_mul(aa, f2_pack(b4.z, b4.w)),
                                      group_part_f32x2<SMALL>(p[4 * c4 + 2], p[4 * c4 + 3]));
          float t0, t1, t2, t3;
          f2_unpack(t01, t0, t1);
          f2_unpack(t23, t2, t3);
          acc[4 * c4] = __fadd_rn(acc[4 * c4], t0);
          acc[4 * c4 + 1] = __fadd_rn(acc[4 * c4 + 1], t1);
          acc[4 * c4 + 2] = __fadd_rn(acc[4 * c4 + 2], t2);
          acc[4 * c4 + 3] = __fadd_rn(acc[4 * c4 + 3], t3);
        }
      }
      {
        // the tile's f32 sums -> TMEM result buffer -> shared epilogue
        const uint32_t oaddr = tmem_addr(tmem_base, quarter * 32, kGOutCol + cbeg);
#pragma unroll
        for (int j = 0; j < kGHalf / 16; ++j) {
          uint32_t r[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(acc[16 * j + e]);
          tmem_st16(oaddr + 16 * j, r);
        }
        tmem_wait_st();
        epi_block<kGBN, false, 1>(tmem_base, kGOutCol, quarter, lane, m0, n0, cbeg, cbeg + kGHalf, M, N, nullptr,
                                  args.out, args.ldo, mode, ep, args.epi_path, &tmC, ebuf, buf);
      }
    }
  fold_done:
    if (args.epi_path == kEpiPathTma && lane == 0) bulk_wait_read<0>();  // sources read: the CTA may leave (stores complete with the grid)
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_after_abort();  // let in-flight TMA / UMMA work retire
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// tmA: int8 activation codes [M, K], tmB: int8 weight codes [N, K], both with
// 128 x 128 boxes and 128-byte swizzle; tmC: the output map (or nullptr for
// the scalar-store epilogue).
int launch_i8g_gemm(int M, int N, int K, int G, const float* a_s, const float* b_st, int ldb, void* out,
                    int out_dtype, const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap* tmC,
                    uint32_t* err, int num_sms, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || G <= 0 || G % 32 || K % G || ldb < ((N + 127) / 128) * 128) return RB_E_SHAPE;
  static uint64_t configured = 0;  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    if (cudaFuncSetAttribute(gemm_i8g_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(gemm_i8g_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGSmem) !=
            cudaSuccess)
      return RB_E_DEVICE;
    configured |= 1ull << (dev & 63);
  }
  GroupArgs a{};
  a.M = M; a.N = N; a.K = K; a.G = G;
  a.a_s = a_s; a.b_st = b_st; a.ldb = ldb;
  a.out = out; a.ldo = N; a.out_dtype = out_dtype; a.err = err;
  a.epi_path = tmC == nullptr ? kEpiPathScalar : epi_path_default();
  const int tiles = ((M + 127) / 128) * ((N + kGBN - 1) / kGBN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  // A programmatic dependent of the group quantiser launched just before it.
  const CUtensorMap& tc = tmC ? *tmC : tmA;
  cudaError_t e;
  if (G <= 256)
    e = launch_kernel(gemm_i8g_kernel<true>, dim3(grid), dim3(kGThreads), kGSmem, stream, true, tmA, tmB, tc, a);
  else
    e = launch_kernel(gemm_i8g_kernel<false>, dim3(grid), dim3(kGThreads), kGSmem, stream, true, tmA, tmB, tc, a);
  if (e != cudaSuccess) return RB_E_DEVICE;
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

}  // namespace rb
