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

#include <atomic>
#include <cstdlib>
#include <cstring>

#include "gemm_common.cuh"

namespace rb {

template <int BN_, int LSTAGES_, int KIND_, int BSTAGES_ = 2, int MH_ = 1>
struct GemmCfg {
  static constexpr int BN = BN_;
  // 128-row M halves per tile: MH = 2 issues two M=128 UMMAs per K step that
  // share one (dequantised) B tile, halving the dequant work per FLOP.
  static constexpr int MH = MH_;
  static constexpr int BM = 128 * MH;
  static constexpr int LSTAGES = LSTAGES_;          // TMA load ring depth
  static constexpr bool I8 = KIND_ == kKindI8;      // int8 UMMA + W8A8 epilogue
  static constexpr bool Q8 = KIND_ == kKindQ8;      // B dequantised from staged codes
  static constexpr bool TMAB = !Q8;                 // B tiles loaded by TMA
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
  static constexpr int EPI_WARPS = I8 ? kNumEpiWarpsI8 : kNumEpiWarps;
  static constexpr int EPI_BUFS = I8 ? 1 : 2;       // staging buffers per epilogue warp
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUFS * kEpiBufBytes;
  static constexpr int BAR_OFF = EPI_OFF + EPI_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 384 + 1024;
  static constexpr int NUM_WARPS = Q8 ? (kDqWarp0 + kNumDqWarps) : kEpiWarp0 + EPI_WARPS;
  static constexpr int THREADS = NUM_WARPS * 32;
  static constexpr int ACC_COLS = MH * BN;          // one accumulator (all M halves)
  static constexpr uint32_t TMEM_COLS = (2 * ACC_COLS <= 32) ? 32 : (2 * ACC_COLS <= 64) ? 64
                                        : (2 * ACC_COLS <= 128) ? 128 : (2 * ACC_COLS <= 256) ? 256 : 512;
  static_assert(2 * ACC_COLS <= 512, "two accumulators must fit in TMEM");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N constraint for M=128");
  static_assert(B_BYTES % 1024 == 0, "B tiles must keep 1024-byte alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

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
      mbar_init(&acc_empty[i], Cfg::EPI_WARPS);
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
    if (args.epi_path == kEpiPathTma) tma_prefetch_desc(&tmC);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // A, row scales and expert tables come from the previous kernel

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one_sync()) {
      int ls = 0;
      uint32_t lph = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        const int m0 = (t / tiles_n) * Cfg::BM;
        int n0 = (t % tiles_n) * BN;
        if (args.tile_expert) {  // grouped: this M tile's weight block starts at expert * N
          const int e = __ldg(args.tile_expert + t / tiles_n);
          if (e < 0) continue;
          n0 += e * N;
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&load_empty[ls], lph ^ 1, args.err, abort_flag)) goto producer_done;
          uint8_t* st = smem + ls * Cfg::LSTAGE;
          mbar_arrive_expect_tx(&load_full[ls], Cfg::LOAD_TX);
          tma_load_2d(st, &tmA, &load_full[ls], kb * Cfg::BK, m0);
          if (Cfg::TMAB) {
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
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        if (args.tile_expert && __ldg(args.tile_expert + t / tiles_n) < 0) continue;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        ++local;  // counts processed tiles only (accumulator ring phases)
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
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + Cfg::EPI_WARPS) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const EpiParams ep{args.s_col, args.out_dtype, args.out_scale, args.out_inv};
    uint8_t* ebuf = smem + Cfg::EPI_OFF + (warp - kEpiWarp0) * Cfg::EPI_BUFS * kEpiBufBytes;
    // With eight epilogue warps, warps 2..5 take the first half of the tile's
    // columns and warps 6..9 the second (each quarter of TMEM lanes has two).
    constexpr int kColSplit = Cfg::EPI_WARPS / 4;
    const int cbeg = ((warp - kEpiWarp0) >> 2) * (BN / kColSplit), cend = cbeg + BN / kColSplit;
    const int mode = args.gated ? kEpiSiluF16 : epi_mode(Cfg::I8, args.out_dtype, args.out_scale, args.act);
    int buf = 0;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      if (args.tile_expert && __ldg(args.tile_expert + t / tiles_n) < 0) continue;
      const int n0 = (t % tiles_n) * BN;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      ++local;
      if (!warp_wait(&acc_full[acc], acc_phase, args.err, abort_flag)) break;
      tc_fence_after();
      for (int h = 0; h < Cfg::MH; ++h) {
      const int m0 = (t / tiles_n) * Cfg::BM + h * 128;
      const uint32_t acc_col = acc * Cfg::ACC_COLS + h * BN;
      epi_block<BN, Cfg::I8, Cfg::EPI_BUFS>(tmem_base, acc_col, quarter, lane, m0, n0, cbeg, cend, M, N,
                                            args.s_row, args.out, args.ldo, mode, ep, args.epi_path,
                                            &tmC, ebuf, buf);
      }  // M halves
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
    if (args.epi_path == kEpiPathTma && lane == 0) bulk_wait_read<0>();  // sources read: the CTA may leave (stores complete with the grid)
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
      if (args.tile_expert && __ldg(args.tile_expert + t / tiles_n) < 0) continue;
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
using CfgQ8_256 = GemmCfg<256, 3, kKindQ8, 2>;
using CfgQ8_128 = GemmCfg<128, 4, kKindQ8, 4>;
using CfgQ8_96 = GemmCfg<96, 4, kKindQ8, 6>;
using CfgQ8_64 = GemmCfg<64, 6, kKindQ8, 6>;
using CfgQ8_128x2 = GemmCfg<128, 3, kKindQ8, 3, 2>;  // 256-row M tile
using CfgI8_256 = GemmCfg<256, 4, kKindI8>;
using CfgI8_128 = GemmCfg<128, 6, kKindI8>;
using CfgF16_256 = GemmCfg<256, 4, kKindF16>;
using CfgF16_128 = GemmCfg<128, 6, kKindF16>;

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
  // Both fast paths write whole 128-byte rows of the N tile; tmC != nullptr
  // means the output rows are 16-byte aligned.
  args.epi_path = (tmC == nullptr || (Cfg::BN % (128 / out_bytes)) != 0) ? kEpiPathScalar
                  : epi_path_default();
  const CUtensorMap& tc = tmC ? *tmC : tmA;
  if (launch_kernel(gemm_kernel<Cfg>, dim3(grid), dim3(Cfg::THREADS), Cfg::SMEM_BYTES, stream, a.pdl != 0,
                    tmA, tmB, tmS, tc, args) != cudaSuccess)
    return RB_E_DEVICE;
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

int epi_path_default() {
  static const int path = [] {
    const char* v = getenv("ROCKET_B200_EPILOGUE");
    if (v && strcmp(v, "tma") == 0) return static_cast<int>(kEpiPathTma);
    if (v && strcmp(v, "vector") == 0) return static_cast<int>(kEpiPathVector);
    return static_cast<int>(kEpiPathTma);  // measured faster on B200 for every GEMM shape
  }();
  return path;
}

static std::atomic<int> g_policy{RB_TILES_AUTO};

int set_gemm_policy(int policy) { return g_policy.exchange(policy); }
int gemm_policy() { return g_policy.load(); }

// Tile plan minimising the makespan of the persistent grid: rounds of tiles
// per SM (per SM pair for the pair kernel) times the per-tile cost. A tile's
// cost is its MMA columns per SM (128-row halves x BN) scaled by a measured
// per-SM efficiency factor of the shape, plus a fixed pipeline fill /
// epilogue overhead. Measured on B200 (rb_matmul, f16 in / out):
//   * W8A8: pair tiles run ~3% faster than single-CTA 128 x 256 tiles at
//     K ~ 1k and ~13% faster at K ~ 4k (per SM they stage and read half the
//     weight bytes; shared-memory bandwidth bounds the single-CTA tile);
//   * Q8_0: pair tiles run ~40% faster than the best single-CTA tile (256 x
//     128, two M halves sharing one dequantised B tile) at large M; at small
//     M (a single round of tiles) the two are even.
GemmPlan gemm_plan(bool i8, int M, int N, int K, int num_sms, bool pair96) {
  const int policy = g_policy.load();
  struct Shape { int bn, mh; bool pair; double eff; };
  const bool long_k = K > 2048;
  // 96-column pair tiles: per SM and k-block ~11% less shared-memory traffic
  // than 128-column ones (A 32 KB + B 18 KB against 32 + 24), which bounds
  // these tiles; they fill 64 SM pairs where 128-column tiles fill 48 at
  // config #1's 512 x 3072.
  const Shape q8c[] = {{256, 1, false, 2.0}, {128, 1, false, 2.0}, {96, 1, false, 2.0},
                       {64, 1, false, 2.0},  {128, 2, false, 1.5}, {256, 1, true, 1.03},
                       {128, 1, true, 1.2},  {96, 1, true, 1.4}};
  const Shape i8c[] = {{256, 1, false, long_k ? 1.13 : 1.04}, {128, 1, false, long_k ? 1.25 : 1.15},
                       {256, 1, true, 1.0}, {128, 1, true, 1.12}};
  const Shape* c = i8 ? i8c : q8c;
  const int nc = i8 ? 4 : (pair96 ? 8 : 7);
  GemmPlan best{c[0].bn, c[0].mh, false};
  double best_cost = -1.0;
  for (int i = 0; i < nc; ++i) {
    if (policy == RB_TILES_SINGLE && c[i].pair) continue;
    if (policy == RB_TILES_PAIR && !c[i].pair) continue;
    const long rows = c[i].pair ? 256L : 128L * c[i].mh;
    const long tiles = ((M + rows - 1) / rows) * ((N + c[i].bn - 1) / c[i].bn);
    const long units = c[i].pair ? num_sms / 2 : num_sms;
    const long rounds = (tiles + units - 1) / units;
    const double cost = rounds * (c[i].mh * c[i].bn * c[i].eff + 32.0);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = GemmPlan{c[i].bn, c[i].mh, c[i].pair};
    }
  }
  return best;
}

static GemmArgs make_args(const GemmLaunch& L) {
  GemmArgs a{};
  a.M = L.M; a.N = L.N; a.K = L.K;
  a.s_row = L.s_row; a.s_col = L.s_col;
  a.out = L.out; a.ldo = L.ldo; a.out_dtype = L.out_dtype;
  a.out_scale = L.out_scale;
  a.out_inv = L.out_scale != 0.0f ? 1.0f / L.out_scale : 0.0f;
  a.err = L.err;
  a.tile_expert = L.tile_expert;
  a.gated = L.gated;
  a.act = L.act;
  a.pdl = L.pdl;
  a.w_codes = L.w_codes;
  a.w_scales = reinterpret_cast<const __half*>(L.w_scales);
  a.w_pitch = L.w_pitch;
  a.w_rows = L.w_rows;
  return a;
}

int launch_q8_gemm_pair(const GemmArgs& a, int bn, int num_sms, const CUtensorMap& tmA,
                        const CUtensorMap& tmCodes, const CUtensorMap& tmScales,
                        const CUtensorMap* tmC, cudaStream_t stream);
int launch_w8a8_gemm_pair(const GemmArgs& a, int bn, int num_sms, const CUtensorMap& tmA,
                          const CUtensorMap& tmB, const CUtensorMap* tmC, cudaStream_t stream);

int launch_q8_gemm(const GemmLaunch& L, const GemmPlan& plan, const CUtensorMap& tmA,
                   const CUtensorMap& tmCodes, const CUtensorMap& tmScales, const CUtensorMap* tmC,
                   cudaStream_t stream) {
  const GemmArgs a = make_args(L);
  if (plan.pair) return launch_q8_gemm_pair(a, plan.bn, L.num_sms, tmA, tmCodes, tmScales, tmC, stream);
  if (plan.mh == 2) {
    if (plan.bn != 128) return RB_E_SHAPE;
    return launch_cfg<CfgQ8_128x2>(tmA, tmCodes, tmScales, tmC, a, L.num_sms, stream);
  }
  switch (plan.bn) {
    case 256: return launch_cfg<CfgQ8_256>(tmA, tmCodes, tmScales, tmC, a, L.num_sms, stream);
    case 128: return launch_cfg<CfgQ8_128>(tmA, tmCodes, tmScales, tmC, a, L.num_sms, stream);
    case 96: return launch_cfg<CfgQ8_96>(tmA, tmCodes, tmScales, tmC, a, L.num_sms, stream);
    case 64: return launch_cfg<CfgQ8_64>(tmA, tmCodes, tmScales, tmC, a, L.num_sms, stream);
    default: return RB_E_SHAPE;
  }
}

int launch_f16_gemm_pair(const GemmArgs& a, int bn, int num_sms, const CUtensorMap& tmA,
                         const CUtensorMap& tmB, const CUtensorMap* tmC, cudaStream_t stream);

int launch_f16_gemm(const GemmLaunch& L, const GemmPlan& plan, const CUtensorMap& tmA,
                    const CUtensorMap& tmB, const CUtensorMap* tmC, cudaStream_t stream) {
  const GemmArgs a = make_args(L);
  if (plan.pair) return launch_f16_gemm_pair(a, plan.bn, L.num_sms, tmA, tmB, tmC, stream);
  switch (plan.bn) {
    case 256: return launch_cfg<CfgF16_256>(tmA, tmB, tmA, tmC, a, L.num_sms, stream);
    case 128: return launch_cfg<CfgF16_128>(tmA, tmB, tmA, tmC, a, L.num_sms, stream);
    default: return RB_E_SHAPE;
  }
}

int launch_w8a8_gemm(const GemmLaunch& L, const GemmPlan& plan, const CUtensorMap& tmA,
                     const CUtensorMap& tmB, const CUtensorMap* tmC, cudaStream_t stream) {
  const GemmArgs a = make_args(L);
  if (plan.pair) return launch_w8a8_gemm_pair(a, plan.bn, L.num_sms, tmA, tmB, tmC, stream);
  switch (plan.bn) {
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
