// gemm_pair.cu — CTA-pair (cta_group::2) tcgen05 GEMMs for large M.
//
// Same two matmul kinds and epilogues as gemm.cu (Q8_0 block-dequant on
// kind::f16, W8A8 on kind::i8), but one output tile of 256 rows x BN columns
// is computed by a pair of CTAs on neighbouring SMs (a (2,1,1) cluster):
//
//   * each CTA stages its own 128 rows of A and its own BN/2 rows of B
//     (int8 codes, or for Q8_0 the codes it dequantises itself);
//   * the leader (cluster rank 0) issues M=256 UMMAs that read A and B from
//     both CTAs' shared memory and write rows 0..127 of the accumulator into
//     the leader's TMEM and rows 128..255 into the peer's;
//   * each CTA's epilogue stores its own 128 rows.
//
// Per SM this halves the B bytes loaded from L2 and read from shared memory
// per FLOP compared with a 128 x BN tile on one SM, which is what bounds the
// single-CTA kernel at large M (L2 -> SM traffic and shared-memory bandwidth),
// and for Q8_0 it halves the dequantisation work per FLOP.
//
// Synchronisation (all waits bounded, see sm100.cuh). A stage holds this
// CTA's 128 rows of A and its half of B (TMA-loaded, or for Q8_0 written by
// the dequant warps), so the UMMA issuer waits once and commits once per
// k-block — its chain of barrier operations is what paces small launches:
//   ld_full[s]   leader only: A (and W8A8 / f16 B) bytes of both CTAs' TMA
//                loads (cta_group::2 loads complete on the leader's barrier);
//                the leader's producer arms it with both CTAs' byte count.
//                Q8_0: also one arrive per warp of the leader's dequant group
//                writing stage s, and one remote arrive from the peer's
//                forwarding thread (warp 1) once the peer's half is written.
//   ld_empty[s]  each CTA: the leader's UMMA commit (multicast to both CTAs);
//                the TMA producer and (Q8_0) the dequant group wait on it.
//   b_local[s]   peer, Q8_0: its dequant group's warps (local arrive), which
//                the forwarding thread waits on. (Cluster-scope arrives are
//                costly: one per stage instead of one per dequant warp.)
// Q8_0 256-column tiles (Cfg::SPLIT) keep the dequantised B halves in a ring
// of their own, so A can run more stages ahead than 32 KB unified stages
// would allow; there the leader's dequant group and the peer's forward arrive
// on b_full[b] instead of ld_full, and the issuer's commit also releases
// b_empty[b] (two waits and two commits per k-block).
//   acc_full[a]  each CTA: the leader's UMMA commit (multicast).
//   acc_local[a] peer: its own epilogue warps (local arrive).
//   acc_empty[a] leader: its own epilogue warps (local arrive) + one remote
//                arrive per tile from the peer's forwarding thread.
#include "gemm_common.cuh"

namespace rb {

// LSTAGES: stages of A + this CTA's B half. Q8_0's dequant warps read the
// weight codes and scales straight from global memory into registers (up to
// DQ_AHEAD stages ahead), so the codes never pass through shared memory,
// whose bandwidth bounds this kernel at large M.
template <int BN_, int LSTAGES_, int KIND_, int DQ_WARPS_ = 8, int DQ_GROUPS_ = 1, int DQ_AHEAD_ = 1,
          int BSTAGES_ = 0>
struct PairCfg {
  static constexpr int DQ_WARPS = DQ_WARPS_;         // Q8_0 dequant warps
  static constexpr int DQ_GROUPS = DQ_GROUPS_;       // stages dequantised concurrently
  // Stages a dequant group's code loads run ahead of the stage it writes.
  // Each group waits a load latency per DQ_AHEAD stages, so weights that
  // come from HBM (small-M launches, a fresh weight per call) want a deeper
  // lookahead than L2-resident ones (large M, each weight tile reused).
  static constexpr int DQ_AHEAD = DQ_AHEAD_;
  static_assert(DQ_WARPS % DQ_GROUPS == 0, "equal dequant groups");
  static constexpr int DQ_GROUP_WARPS = DQ_WARPS / DQ_GROUPS;
  static constexpr int BN = BN_;                    // UMMA N of the pair tile
  static constexpr int HB = BN / 2;                 // weight rows staged per CTA
  static constexpr int LSTAGES = LSTAGES_;
  static constexpr bool I8 = KIND_ == kKindI8;
  static constexpr bool Q8 = KIND_ == kKindQ8;
  static constexpr bool TMAB = !Q8;                 // B halves loaded by TMA
  static constexpr int ELEM = I8 ? 1 : 2;
  static constexpr int BK = 128 / ELEM;             // K elements per stage (one 128-B atom)
  static constexpr int UMMA_K = I8 ? 32 : 16;
  static constexpr int KSTEPS = BK / UMMA_K;        // 4
  static constexpr int A_BYTES = 128 * 128;         // this CTA's 128 rows of A
  static constexpr int B_BYTES = HB * 128;          // this CTA's half of B (s8, or dequantised f16)
  static constexpr uint32_t PAIR_TX = TMAB ? 2 * (A_BYTES + B_BYTES) : 2 * A_BYTES;
  // Q8_0 with BSTAGES_ > 0: the dequantised B halves live in a ring of their
  // own, so A can run LSTAGES stages ahead while B runs BSTAGES (256-column
  // tiles: a 32 KB unified stage would leave room for 6 stages of each).
  static constexpr bool SPLIT = Q8 && BSTAGES_ > 0;
  static constexpr int NB = SPLIT ? BSTAGES_ : LSTAGES;  // B slots (and b_local entries)
  static constexpr int LSTAGE = round1k(A_BYTES + (SPLIT ? 0 : B_BYTES));
  static constexpr int BRING_OFF = LSTAGES * LSTAGE;
  static constexpr int EPI_OFF = BRING_OFF + (SPLIT ? NB * B_BYTES : 0);
  static constexpr int EPI_WARPS = I8 ? kNumEpiWarpsI8 : kNumEpiWarps;
  static constexpr int EPI_BUFS = 1;                // staging buffers per epilogue warp
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUFS * kEpiBufBytes;
  static constexpr int BAR_OFF = EPI_OFF + EPI_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 512 + 1024;
  // After the role warps: the peer's accumulator-release forwarder (idle in
  // the leader).
  static constexpr int FWD_WARP = Q8 ? (kDqWarp0 + DQ_WARPS) : kEpiWarp0 + EPI_WARPS;
  static constexpr int NUM_WARPS = FWD_WARP + 1;
  static constexpr int THREADS = NUM_WARPS * 32;
  // Two accumulators, the second at a 128- or 256-column boundary (BN = 96
  // tiles leave 32 columns of each 128 unused).
  static constexpr uint32_t ACC_STRIDE = BN <= 128 ? 128 : 256;
  static constexpr uint32_t TMEM_COLS = 2 * ACC_STRIDE;
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "pair UMMA N");
  static_assert(B_BYTES % 1024 == 0, "B halves keep 1024-byte alignment");
  static_assert(BAR_OFF % 1024 == 0 && A_BYTES % 1024 == 0, "stage alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

template <class Cfg>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg::THREADS, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmC,
                 GemmArgs args) {
  constexpr int BN = Cfg::BN;
  constexpr int HB = Cfg::HB;
  constexpr int LSTAGES = Cfg::LSTAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t* ld_full = bars;                          // [LSTAGES]
  uint64_t* ld_empty = ld_full + LSTAGES;            // [LSTAGES]
  uint64_t* b_local = ld_empty + LSTAGES;            // [NB] (Q8_0 peer)
  uint64_t* b_full = b_local + Cfg::NB;              // [NB] (split Q8_0 rings, leader)
  uint64_t* b_empty = b_full + Cfg::NB;              // [NB] (split Q8_0 rings)
  uint64_t* acc_full = b_empty + Cfg::NB;            // [2]
  uint64_t* acc_empty = acc_full + 2;                // [2]
  uint64_t* acc_local = acc_empty + 2;               // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_local + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int M = args.M, N = args.N, K = args.K;
  const int tiles_n = (N + BN - 1) / BN;
  const int tiles_m = (M + 255) / 256;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + Cfg::BK - 1) / Cfg::BK;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  // Grouped GEMM (tile_expert != nullptr): the first weight row of tile t's
  // expert block. Expert segments are 256-row aligned, so both 128-row
  // halves of a pair tile share one expert (entries are per 128 rows); the
  // tiles past the used segments (-1) form a suffix of the tile order, and
  // every role stops at the first of them, so all roles see the same tiles.
  auto expert_row0 = [&](int t) -> int {
    if (!args.tile_expert) return 0;
    const int e = __ldg(args.tile_expert + 2 * (t / tiles_n));
    return e < 0 ? -1 : e * N;
  };

  // Q8_0 pairs with exactly one tile (small M, e.g. a 512-row call): once
  // that tile's main loop is done the dequant warps have nothing left to do,
  // so they drain the accumulator beside the epilogue warps, each warp of a
  // TMEM lane quarter taking a column slice (the stage ring, read by no UMMA
  // any more, serves as their staging). Not for the gated epilogue, whose chunks
  // span 128 accumulator columns.
  const int epi_mode_k = args.gated ? kEpiSiluF16 : epi_mode(Cfg::I8, args.out_dtype, args.out_scale, args.act);
  const int epi_cw = (epi_mode_k == kEpiRaw4) ? 32 : 64;  // columns per epilogue chunk (Q8_0 modes)
  const int help_slices = BN / epi_cw < 4 ? BN / epi_cw : 4;
  const bool one_tile = Cfg::Q8 && Cfg::DQ_WARPS == 12 && !args.gated && args.tile_expert == nullptr &&
                        num_tiles <= npairs && pair < num_tiles && help_slices > 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < LSTAGES; ++s) {
      // Q8_0 leader: the producer's expect-tx arrive, its dequant group's
      // warps and the peer's forwarded arrive.
      mbar_init(&ld_full[s], Cfg::Q8 && !Cfg::SPLIT ? Cfg::DQ_GROUP_WARPS + 2 : 1);
      mbar_init(&ld_empty[s], 1);
    }
    for (int s = 0; s < Cfg::NB; ++s) {
      mbar_init(&b_local[s], Cfg::DQ_GROUP_WARPS);
      // split rings, leader: its dequant group's warps and the peer's forward
      mbar_init(&b_full[s], Cfg::DQ_GROUP_WARPS + 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], Cfg::EPI_WARPS + 1);
      mbar_init(&acc_local[i], Cfg::EPI_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (args.epi_path == kEpiPathTma) tma_prefetch_desc(&tmC);
  }
  // ------------------------------------------------------------ Q8_0 dequant role: layout and first loads
  constexpr int kGroupWarps = Cfg::DQ_WARPS / Cfg::DQ_GROUPS;
  constexpr int kThreads = kGroupWarps * 32;
  constexpr int kRowStep = kThreads / 8;
  constexpr int kPer = HB / kRowStep;
  static_assert(HB % kRowStep == 0, "whole chunks per thread");
  const bool dq_warp = Cfg::Q8 && warp >= kDqWarp0 && warp < kDqWarp0 + Cfg::DQ_WARPS;
  const int grp = dq_warp ? (warp - kDqWarp0) / kGroupWarps : 0;
  const int tid = threadIdx.x - (kDqWarp0 + grp * kGroupWarps) * 32;
  const int c = tid & 7, r0 = tid >> 3;
  const int8_t* __restrict__ wc = args.w_codes;
  const __half* __restrict__ ws = args.w_scales;
  struct Staged {
    uint2 q[kPer];
    __half d[kPer];
  };
  // Stage q of the sequence is k-block q % num_kb of this pair's tile
  // number q / num_kb; false past the last tile.
  auto fetch = [&](int q, Staged& st) -> bool {
    const int t = pair + (q / num_kb) * npairs;
    if (t >= num_tiles) return false;
    const int w0 = expert_row0(t);
    if (w0 < 0) return false;
    const int kb = q % num_kb;
    const long long row0 = static_cast<long long>(w0) + (t % tiles_n) * BN + static_cast<int>(rank) * HB + r0;
    const int col = kb * 64 + c * 8;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const long long row = row0 + j * kRowStep;
      if (row < args.w_rows && col < K) {
        st.q[j] = __ldg(reinterpret_cast<const uint2*>(wc + row * K + col));
        st.d[j] = ws[static_cast<long long>(col >> 5) * args.w_pitch + row];
      } else {
        st.q[j] = make_uint2(0u, 0u);
        st.d[j] = __ushort_as_half(0);
      }
    }
    return true;
  };
  // st[i] holds the group's stage q + i * DQ_GROUPS (q: the stage it
  // writes next). The dequant warps issue their first DQ_AHEAD stages' loads
  // before the set-up barrier, so a cold weight's HBM latency overlaps the
  // set-up (and, under programmatic dependent launch, the previous kernel);
  // they arrive on that barrier with relaxed semantics (they have written
  // nothing to publish), which does not wait for those loads to complete.
  // Grouped GEMMs first need the expert table, which the previous kernel
  // writes: they load after griddepcontrol.wait.
  Staged st[Cfg::DQ_AHEAD + 1];
  bool hv[Cfg::DQ_AHEAD + 1];
#pragma unroll
  for (int i = 0; i <= Cfg::DQ_AHEAD; ++i) hv[i] = false;
  const bool dq_early = dq_warp && args.tile_expert == nullptr;
  if (dq_early) {
#pragma unroll
    for (int i = 0; i < Cfg::DQ_AHEAD; ++i) hv[i] = fetch(grp + i * Cfg::DQ_GROUPS, st[i]);
  }

  // Both CTAs' barriers are initialised (and visible cluster-wide) before any
  // TMA completion or remote arrive can target them.
  tc_fence_before();
  if (dq_early) cluster_sync_relaxed_arrive();
  else cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // A, row scales and expert tables come from the previous kernel; the Q8_0
  // dequant warps read only the resident weight, and start on it at once
  // unless they need the expert table.
  if (!(Cfg::Q8 && args.tile_expert == nullptr && warp >= kDqWarp0)) griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (elect_one_sync()) {
      int ls = 0;
      uint32_t lph = 0;
      for (int t = pair; t < num_tiles; t += npairs) {
        const int w0 = expert_row0(t);
        if (w0 < 0) break;
        const int m0 = (t / tiles_n) * 256 + static_cast<int>(rank) * 128;
        const int nb = w0 + (t % tiles_n) * BN + static_cast<int>(rank) * HB;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&ld_empty[ls], lph ^ 1, args.err, abort_flag)) goto producer_done;
          uint8_t* st = smem + ls * Cfg::LSTAGE;
          const uint32_t lf = mapa_shared(&ld_full[ls], 0);
          if (rank == 0) mbar_arrive_expect_tx(&ld_full[ls], Cfg::PAIR_TX);
          tma_load_2d_pair(st, &tmA, lf, kb * Cfg::BK, m0);
          if constexpr (Cfg::TMAB) tma_load_2d_pair(st + Cfg::A_BYTES, &tmB, lf, kb * Cfg::BK, nb);
          if (++ls == LSTAGES) { ls = 0; lph ^= 1; }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer (leader)
    if (rank == 0 && elect_one_sync()) {
      constexpr uint32_t idesc =
          Cfg::I8 ? idesc_i8(256, BN) : idesc_f16(256, BN, false, false, false);
      constexpr uint16_t kBoth = 0x3;
      int ls = 0, bs = 0;
      uint32_t lph = 0, bph = 0;
      int local = 0;
      for (int t = pair; t < num_tiles; t += npairs, ++local) {
        if (expert_row0(t) < 0) break;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_cluster(&acc_empty[acc], acc_phase ^ 1, args.err, abort_flag)) goto mma_done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * Cfg::ACC_STRIDE;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_cluster(&ld_full[ls], lph, args.err, abort_flag)) goto mma_done;
          if constexpr (Cfg::SPLIT) {
            if (!mbar_wait_cluster(&b_full[bs], bph, args.err, abort_flag)) goto mma_done;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + ls * Cfg::LSTAGE);
          const uint32_t b_addr = Cfg::SPLIT ? smem_u32(smem + Cfg::BRING_OFF + bs * Cfg::B_BYTES)
                                             : a_addr + Cfg::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < Cfg::KSTEPS; ++ks) {
            const uint64_t da = desc_kmajor_sw128(a_addr + ks * 32);
            const uint64_t db = desc_kmajor_sw128(b_addr + ks * 32);
            const uint32_t accum = (kb > 0 || ks > 0) ? 1u : 0u;
            if constexpr (Cfg::I8) umma_i8_pair(d_tmem, da, db, idesc, accum);
            else umma_f16_pair(d_tmem, da, db, idesc, accum);
          }
          umma_commit_pair(&ld_empty[ls], kBoth);  // both CTAs' stage s is free once these retire
          if (++ls == LSTAGES) { ls = 0; lph ^= 1; }
          if constexpr (Cfg::SPLIT) {
            umma_commit_pair(&b_empty[bs], kBoth);
            if (++bs == Cfg::NB) { bs = 0; bph ^= 1; }
          }
        }
        umma_commit_pair(&acc_full[acc], kBoth);
      }
    mma_done:;
    } else if (rank == 1 && Cfg::Q8 && elect_one_sync()) {
      // Peer: forward "my half of B in slot bs is written" to the leader's
      // ld_full (b_full with split rings), once per stage.
      int bs = 0;
      uint32_t bph = 0;
      for (int t = pair; t < num_tiles; t += npairs) {
        if (expert_row0(t) < 0) break;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&b_local[bs], bph, args.err, abort_flag)) goto fwd_b_done;
          mbar_arrive_cluster(mapa_shared(Cfg::SPLIT ? &b_full[bs] : &ld_full[bs], 0));
          if (++bs == Cfg::NB) { bs = 0; bph ^= 1; }
        }
      }
    fwd_b_done:;
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + Cfg::EPI_WARPS) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const EpiParams ep{args.s_col, args.out_dtype, args.out_scale, args.out_inv};
    uint8_t* ebuf = smem + Cfg::EPI_OFF + (warp - kEpiWarp0) * Cfg::EPI_BUFS * kEpiBufBytes;
    constexpr int kColSplit = Cfg::EPI_WARPS / 4;  // warps sharing a TMEM lane quarter
    int cbeg = ((warp - kEpiWarp0) >> 2) * (BN / kColSplit), cend = cbeg + BN / kColSplit;
    if (one_tile) {  // slice 0 of the quarter's columns; dequant warps take the others
      cbeg = 0;
      cend = BN / help_slices;
    }
    const int mode = epi_mode_k;
    int buf = 0;
    int local = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++local) {
      if (expert_row0(t) < 0) break;
      const int n0 = (t % tiles_n) * BN;
      const int m0 = (t / tiles_n) * 256 + static_cast<int>(rank) * 128;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!warp_wait(&acc_full[acc], acc_phase, args.err, abort_flag)) break;
      tc_fence_after();
      epi_block<BN, Cfg::I8, Cfg::EPI_BUFS>(tmem_base, acc * Cfg::ACC_STRIDE, quarter, lane, m0, n0, cbeg, cend, M, N,
                                            args.s_row, args.out, args.ldo, mode, ep, args.epi_path,
                                            &tmC, ebuf, buf);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(rank == 0 ? &acc_empty[acc] : &acc_local[acc]);
    }
    if (args.epi_path == kEpiPathTma && lane == 0) bulk_wait_read<0>();  // sources read: the CTA may leave (stores complete with the grid)
  } else if (warp == Cfg::FWD_WARP) {
    // ------------------------------------------------------------ peer: accumulator release
    // Forward "my accumulator rows are drained" to the leader, once per tile.
    if (rank == 1 && elect_one_sync()) {
      int local = 0;
      for (int t = pair; t < num_tiles; t += npairs, ++local) {
        if (expert_row0(t) < 0) break;
        const int acc = local & 1;
        if (!mbar_wait(&acc_local[acc], (local >> 1) & 1, args.err, abort_flag)) break;
        mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
      }
    }
  } else if (Cfg::Q8 && warp >= kDqWarp0) {
    // ------------------------------------------------------------ Q8_0 dequant (both CTAs)
    // The dequant warps form DQ_GROUPS groups; group g dequantises stages
    // q = g, g + DQ_GROUPS, ... of the (tile, k-block) sequence, so several
    // stages are in flight at once. Thread `tid` of a group owns the chunks
    // (row r0 + j * kRowStep, column c): 8 codes of one of this CTA's HB
    // weight rows and their block's f16 scale. It loads them for the group's
    // stage DQ_AHEAD ahead from global memory (read-only path; L2 after the
    // first M tile) before it writes the current stage as 8 f16 values per chunk in
    // the 128-byte swizzled K-major layout the UMMA descriptor reads. Rows
    // past the weight and columns past K read as zero (the TMA fill).
    if (!dq_early) {
#pragma unroll
      for (int i = 0; i < Cfg::DQ_AHEAD; ++i) hv[i] = fetch(grp + i * Cfg::DQ_GROUPS, st[i]);
    }
    int q = grp;
    while (hv[0]) {
      // in flight while this stage and the next DQ_AHEAD - 1 are written
      hv[Cfg::DQ_AHEAD] = fetch(q + Cfg::DQ_AHEAD * Cfg::DQ_GROUPS, st[Cfg::DQ_AHEAD]);
      const int bs = q % Cfg::NB;
      const uint32_t bph = (q / Cfg::NB) & 1;
      if (!warp_wait(Cfg::SPLIT ? &b_empty[bs] : &ld_empty[bs], bph ^ 1, args.err, abort_flag)) goto dq_done;
      uint8_t* sb = Cfg::SPLIT ? smem + Cfg::BRING_OFF + bs * Cfg::B_BYTES : smem + bs * Cfg::LSTAGE + Cfg::A_BYTES;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int rowi = r0 + j * kRowStep;
        *reinterpret_cast<uint4*>(sb + rowi * 128 + ((c ^ (rowi & 7)) << 4)) =
            q8_dequant8_f16(st[0].q[j], st[0].d[j]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0)  // this CTA's half of B is written
        mbar_arrive(rank != 0 ? &b_local[bs] : (Cfg::SPLIT ? &b_full[bs] : &ld_full[bs]));
#pragma unroll
      for (int i = 0; i < Cfg::DQ_AHEAD; ++i) {
        st[i] = st[i + 1];
        hv[i] = hv[i + 1];
      }
      q += Cfg::DQ_GROUPS;
    }
    // Single-tile pair: help drain the accumulator (slices 1.. of this warp's
    // lane quarter; three dequant warps per quarter).
    if (one_tile && (warp - kDqWarp0) / 4 + 1 < help_slices) {
      const int slice = (warp - kDqWarp0) / 4 + 1;
      if (!warp_wait(&acc_full[0], 0, args.err, abort_flag)) goto dq_done;
      tc_fence_after();
      const EpiParams ep{args.s_col, args.out_dtype, args.out_scale, args.out_inv};
      uint8_t* ebuf = smem + (warp - kDqWarp0) * kEpiBufBytes;  // in the drained stage ring
      int buf = 0;
      const int w = BN / help_slices;
      epi_block<BN, false, 1>(tmem_base, 0, warp & 3, lane, (pair / tiles_n) * 256 + static_cast<int>(rank) * 128,
                              (pair % tiles_n) * BN, slice * w, (slice + 1) * w, M, N, args.s_row, args.out,
                              args.ldo, epi_mode_k, ep, args.epi_path, &tmC, ebuf, buf);
      if (args.epi_path == kEpiPathTma && lane == 0) bulk_wait_read<0>();  // sources read: the CTA may leave (stores complete with the grid)
    }
  dq_done:;
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_after_abort();  // let in-flight TMA / UMMA work retire
  // Neither CTA leaves (or frees TMEM) while the pair's UMMAs may still read
  // its shared memory or write its TMEM.
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

// --------------------------------------------------------------------------
// Host-side launch.

using PairQ8_256 = PairCfg<256, 7, kKindQ8, 12, 3, 1, 6>;
// 128- and 96-column tiles serve small M (config #1: each call a fresh
// weight from HBM): code loads three stages ahead per group.
using PairQ8_128 = PairCfg<128, 8, kKindQ8, 12, 3, 3>;
using PairQ8_96 = PairCfg<96, 9, kKindQ8, 12, 3, 3>;
using PairI8_256 = PairCfg<256, 6, kKindI8>;
using PairI8_128 = PairCfg<128, 8, kKindI8>;
using PairF16_256 = PairCfg<256, 6, kKindF16>;
using PairF16_128 = PairCfg<128, 8, kKindF16>;

template <class Cfg>
static int launch_pair_cfg(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmS,
                           const CUtensorMap* tmC, const GemmArgs& a, int num_sms,
                           cudaStream_t stream) {
  const int tiles = ((a.M + 255) / 256) * ((a.N + Cfg::BN - 1) / Cfg::BN);
  static uint64_t configured = 0;  // one bit per device ordinal
  static int max_pairs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    if (cudaFuncSetAttribute(gemm_pair_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg::SMEM_BYTES) != cudaSuccess)
      return RB_E_DEVICE;
    // Co-resident pairs: one CTA per SM, two SMs of a cluster-capable pair.
    // (The kernel's compile-time cluster shape applies; none is passed here.)
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * (num_sms / 2));
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_pair_kernel<Cfg>, &cfg) != cudaSuccess ||
        clusters < 1) {
      cudaGetLastError();
      clusters = num_sms / 2;
    }
    max_pairs[dev & 63] = clusters;
    configured |= 1ull << (dev & 63);
  }
  int pairs = max_pairs[dev & 63];
  if (pairs > tiles) pairs = tiles;
  GemmArgs args = a;
  const int out_bytes = (a.out_dtype == RB_DTYPE_F16 || a.out_dtype == RB_DTYPE_BF16) ? 2 : 4;
  // Both fast paths write whole 128-byte rows of the N tile; tmC != nullptr
  // means the output rows are 16-byte aligned.
  args.epi_path = (tmC == nullptr || (Cfg::BN % (128 / out_bytes)) != 0) ? kEpiPathScalar
                  : epi_path_default();
  const CUtensorMap& tc = tmC ? *tmC : tmA;
  if (launch_kernel(gemm_pair_kernel<Cfg>, dim3(2 * pairs), dim3(Cfg::THREADS), Cfg::SMEM_BYTES, stream,
                    a.pdl != 0, tmA, tmB, tmS, tc, args) != cudaSuccess)
    return RB_E_DEVICE;
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

int launch_q8_gemm_pair(const GemmArgs& a, int bn, int num_sms, const CUtensorMap& tmA,
                        const CUtensorMap& tmCodes, const CUtensorMap& tmScales,
                        const CUtensorMap* tmC, cudaStream_t stream) {
  switch (bn) {
    case 256: return launch_pair_cfg<PairQ8_256>(tmA, tmCodes, tmScales, tmC, a, num_sms, stream);
    case 128: return launch_pair_cfg<PairQ8_128>(tmA, tmCodes, tmScales, tmC, a, num_sms, stream);
    case 96: return launch_pair_cfg<PairQ8_96>(tmA, tmCodes, tmScales, tmC, a, num_sms, stream);
    default: return RB_E_SHAPE;
  }
}

int launch_f16_gemm_pair(const GemmArgs& a, int bn, int num_sms, const CUtensorMap& tmA,
                         const CUtensorMap& tmB, const CUtensorMap* tmC, cudaStream_t stream) {
  switch (bn) {
    case 256: return launch_pair_cfg<PairF16_256>(tmA, tmB, tmA, tmC, a, num_sms, stream);
    case 128: return launch_pair_cfg<PairF16_128>(tmA, tmB, tmA, tmC, a, num_sms, stream);
    default: return RB_E_SHAPE;
  }
}

int launch_w8a8_gemm_pair(const GemmArgs& a, int bn, int num_sms, const CUtensorMap& tmA,
                          const CUtensorMap& tmB, const CUtensorMap* tmC, cudaStream_t stream) {
  switch (bn) {
    case 256: return launch_pair_cfg<PairI8_256>(tmA, tmB, tmA, tmC, a, num_sms, stream);
    case 128: return launch_pair_cfg<PairI8_128>(tmA, tmB, tmA, tmC, a, num_sms, stream);
    default: return RB_E_SHAPE;
  }
}

}  // namespace rb
