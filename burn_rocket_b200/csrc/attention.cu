// attention.cu — fused masked grouped-query flash attention for sm_100a.
//
// Semantics: crates/rocket-npu/src/attn/oneshot.rs:130-199 (flash_attn_ref +
// fa_score) with the mask predicates of crates/burn-rocket/src/masks.rs:11-114
// evaluated in-kernel instead of an [n_q, n_kv] additive mask:
//   s   = qk * scale;  s = softcap * tanh(s / softcap) when softcap != 0
//   s   = max(s + mask, -30000)     (mask = 0 visible, -inf hidden)
//   out = sum_j exp(s_j - max) v_j / sum_j exp(s_j - max)   over the real keys
// so a fully masked row averages the values of every key it iterates, as the
// reference does.
//
// Design (a work unit = two 128-row query "slots" sharing one KV head):
//   * GQA: the two slots are two query heads of one KV group (or two query
//     tiles of one head when the group has a single head), so every K/V tile
//     is loaded by TMA once and consumed by both slots.
//   * warp 0: TMA (Q per unit, then K and V rings of 128-key tiles, 128-B
//     swizzled); warp 1: UMMA issuer; warps 2-5 / 6-9: softmax of slot 0 /
//     slot 1, one query row per thread (TMEM lane = row).
//   * TMEM per slot (256 columns): S, a 128 x 128 f32 score tile (M=128,
//     N=128 UMMAs: the shape that runs the tensor pipe at its full rate from
//     shared-memory operands), and O in D columns. P = exp2(S - m) is written
//     back as packed f16/bf16 over the first 64 columns of S and consumed by a
//     TS-form UMMA (A from TMEM) O += P·V.
//   * One S buffer per slot, the two slots in ping-pong: per key tile the
//     UMMA warp issues slot 0's P·V(j) and S(j+1), then slot 1's, so the
//     tensor pipe works on one slot while the other slot's softmax runs. A
//     slot's S(j+1) is issued behind its own P·V(j), so its commit also
//     retires P·V(j): the softmax may rescale O without a separate wait.
//   * Schedules: one CTA per unit, or (split) one CTA per SM over an equal
//     share of all units' key tiles, units cut at share boundaries being
//     merged by whichever part finishes last (see launch_attention).
//   * Online softmax in the log2 domain with a lazy rescale: the exponent base
//     only moves (and O, l are rescaled) when a new row max exceeds it by more
//     than 8 (a factor 256), so P stays within f16 range and O is rarely
//     touched by the softmax warps.
//   * The -30000 clamp is exact: once a row's exponent base lies 160 above the
//     clamp (any row with a visible key scoring above ~-29900), every clamped
//     or masked key underflows to 0 either way, and the warp takes the fast
//     path (one FFMA + one MUFU ex2 per score).
//   * Causal / window / block masks: the visible keys of a row form one
//     interval; key tiles wholly outside a slot's visible band are skipped,
//     tiles wholly inside skip the predicate, and a slot that may contain a
//     fully masked row iterates every key tile.
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "sm100.cuh"
#include "kernels.h"

#include <algorithm>
#include <atomic>
#include <queue>
#include <vector>

namespace rb {

namespace attn {

constexpr int BM = 128;      // query rows per slot
constexpr int BN = kAttnKeyTile;    // keys per tile (128)
#ifndef RB_ATTN_POLY_EVERY
#define RB_ATTN_POLY_EVERY 4  // every 4th pair of scores: exp2 by polynomial
#endif
constexpr int kSoftWarp0 = 2;       // warps 2-5: slot 0, warps 6-9: slot 1
constexpr int kThreads = 10 * 32;   // 3 warps on some SM sub-partitions: 168 registers a thread
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kClamp = -30000.0f;   // fa_score clamp (oneshot.rs PAD_KEY_SCORE)
constexpr float kClamp2 = kClamp * kLog2e;
constexpr float kRescaleThresh = 8.0f;  // log2 units
constexpr float kFastMargin = 160.0f;   // exp2(-160) underflows f32 to 0
constexpr int kNoBound = 1 << 30;
constexpr int kMaxCtas = kAttnMaxCtas;  // split-mode grid bound (>= SM count)
// Split-mode planning: each unit is charged kItemCost key tiles on top of
// its own when the shares are cut (one 128-key tile ~ 1.2 us of a CTA's time).
constexpr int kItemCost = 3;
// Schedule choice, in key tiles, fitted to measured runs (config #2 both
// masks, 64 x 512 and 4 x 2048 token batches, 16 x 2394 at head_dim 72):
constexpr double kCtaTime = 2.5;    // one CTA per unit: a CTA's launch, prologue and epilogue
constexpr double kItemTime = 1.5;   // split: one more item in a CTA's walk
constexpr double kMergeTime = 5.0;  // split: a CTA's partial records and merges

std::atomic<int> g_split_policy{RB_ATTN_SPLIT_AUTO};

struct Params {
  void* out;
  int n_q, n_kv, n_head, n_kv_heads, group;
  int ldo;
  int q_tiles;
  int pairs_per_group;
  float scale_log2;    // scale * log2(e)
  float scale;
  float softcap;
  int dlo, dhi;        // visible iff dlo <= (k_off + j) - (q_off + i) <= dhi
  int q_off, k_off;
  int d_out;           // output columns per head (<= D: the real head_dim)
  int head3d;          // maps are [rows, heads, d_out] views: coordinates (column, head, row)
  // Sequences lie back to back: sequence b owns query rows [b*n_q, (b+1)*n_q)
  // and key rows [b*n_kv, (b+1)*n_kv) of the tensors.
  int batch;
  int n_units;         // batch * pairs_per_group * n_kv_heads work units
  // Split mode (split != 0): G CTAs share the W cost positions of all units
  // evenly (SplitPlan gives each CTA's starting unit).
  int split, W, G;
  int item_cost;       // cost positions charged per unit on top of its key tiles
  float* rec;          // [G][2 records][2 slots] partial (O, m, l)
  int* cnt;            // [n_units][2 slots] parts arrived (self-resetting)
  uint32_t* err;
};

// Split mode: CTA c starts inside unit u0[c], whose first cost position is
// pre0[c]. A separate grid-constant parameter, so that the per-tile reads of
// Params stay plain constant-bank operands.
struct SplitPlan {
  int u0[kMaxCtas];
  int pre0[kMaxCtas];
};

// A head row of D elements is staged as D/64 128-byte-swizzled atoms of 64
// columns plus, when D % 64 == 16 (D = 80: head_dim 72 zero-padded to the
// UMMA K granularity), one 32-byte-swizzled tail atom of 16 columns.
template <int D>
struct Smem {
  static constexpr int ATOMS = D / 64;              // 64-element (128-B) column atoms
  static constexpr int TAIL = D % 64;               // 0 or 16 columns (32-B rows)
  static_assert(TAIL == 0 || TAIL == 16, "head width must be 64k or 64k+16");
  static constexpr int Q_ATOM = BM * 128;           // 16 KB
  static constexpr int KV_ATOM = BN * 128;          // 16 KB
  static constexpr int Q_TAIL_OFF = ATOMS * Q_ATOM;
  static constexpr int KV_TAIL_OFF = ATOMS * KV_ATOM;
  static constexpr int Q_TILE = ATOMS * Q_ATOM + BM * TAIL * 2;
  static constexpr int KV_TILE = ATOMS * KV_ATOM + BN * TAIL * 2;
  static_assert(Q_TILE % 1024 == 0 && KV_TILE % 1024 == 0, "tiles keep 1024-B alignment");
  // K and V rings fill what the two Q tiles leave of the 227 KB (D = 128:
  // 3 K + 2 V stages; narrower heads: 4 + 4).
  static constexpr int FREE = 232448 - 512 - 1024 - 2 * Q_TILE;
  static constexpr int NKV = FREE / KV_TILE;
  static constexpr int V_STAGES = NKV / 2 > 4 ? 4 : NKV / 2;
  static constexpr int K_STAGES = NKV - V_STAGES > 4 ? 4 : NKV - V_STAGES;
  static_assert(K_STAGES >= 2 && V_STAGES >= 2, "K/V double buffering");
  static constexpr int Q_OFF = 0;                   // 2 slots
  static constexpr int K_OFF = 2 * Q_TILE;
  static constexpr int V_OFF = K_OFF + K_STAGES * KV_TILE;
  static constexpr int BAR_OFF = V_OFF + V_STAGES * KV_TILE;
  static constexpr int BYTES = BAR_OFF + 512 + 1024;
  static_assert(BYTES <= 232448, "shared memory budget");
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp2 of a pair of scores on the FMA/ALU pipes, used for every
// kPolyEvery-th pair of the unmasked fast path so that the MUFU pipe (one
// ex2 per score otherwise, 16 a clock per SM: as many cycles per key tile as
// the tile's UMMAs at head_dim 128) does not bound the softmax. Range
// reduction y = j + f with j = floor(y): 1.5 * 2^23 + y rounded toward -inf
// is exact and holds j in its low mantissa bits, whose shift by 23 adds j to
// the exponent field. 2^f on [0, 1) is a degree-3 polynomial fitted for the
// least maximum relative error (Lawson's iteratively reweighted least
// squares): 7.5e-5 relative, below half an ulp of the f16 P it becomes. y is
// clamped at -126: smaller scores round to 0 in an f16/bf16 P either way.
constexpr int kPolyEvery = RB_ATTN_POLY_EVERY;
// Only at head_dim 128, where the exponentials cost as many MUFU cycles as
// the tile's UMMAs: at the narrower widths (64, 72 staged as 80) the
// polynomial measured slower than MUFU alone (config #4's attention 902
// against 866 us).
template <int D>
constexpr int poly_every() { return D >= 128 ? kPolyEvery : 0; }
constexpr float kPolyC0 = 0.9999251365661621f, kPolyC1 = 0.6958339810371399f,
                kPolyC2 = 0.22606706619262695f, kPolyC3 = 0.07802402973175049f;

__device__ __forceinline__ void exp2_poly2(float y0, float y1, float& p0, float& p1) {
  const uint64_t y = f2_pack(fmaxf(y0, -126.0f), fmaxf(y1, -126.0f));
  const uint64_t t = f2_add_rm(y, f2_pack(12582912.0f, 12582912.0f));
  const uint64_t j = f2_add(t, f2_pack(-12582912.0f, -12582912.0f));  // floor(y), exact
  const uint64_t f = f2_fma(j, f2_pack(-1.0f, -1.0f), y);              // y - floor(y), exact
  uint64_t q = f2_fma(f2_pack(kPolyC3, kPolyC3), f, f2_pack(kPolyC2, kPolyC2));
  q = f2_fma(q, f, f2_pack(kPolyC1, kPolyC1));
  q = f2_fma(q, f, f2_pack(kPolyC0, kPolyC0));
  float q0, q1, t0, t1;
  f2_unpack(q, q0, q1);
  f2_unpack(t, t0, t1);
  p0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
  p1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

struct SlotInfo {
  int head;   // query head
  int qt;     // query tile
  int lo, hi; // key tile range (inclusive); empty when lo > hi
};

__host__ __device__ __forceinline__ long lmax_(long a, long b) { return a > b ? a : b; }
__host__ __device__ __forceinline__ long lmin_(long a, long b) { return a < b ? a : b; }

__host__ __device__ inline SlotInfo slot_info(const Params& p, int g, int item) {
  SlotInfo s;
  const int total = p.group * p.q_tiles;
  if (item >= total) { s.head = 0; s.qt = 0; s.lo = 1; s.hi = 0; return s; }
  s.qt = item / p.group;
  s.head = g * p.group + item % p.group;
  const int n_kv_tiles = (p.n_kv + BN - 1) / BN;
  const int qa0 = p.q_off + s.qt * BM;
  const int qa1 = p.q_off + static_cast<int>(lmin_(s.qt * BM + BM, p.n_q)) - 1;
  // Visible absolute keys of row qa: [qa + dlo, qa + dhi] ∩ [k_off, k_off + n_kv).
  const long klast = static_cast<long>(p.k_off) + p.n_kv - 1;
  auto row_empty = [&](int qa) {
    const long lo = (p.dlo <= -kNoBound) ? p.k_off : lmax_(static_cast<long>(p.k_off), static_cast<long>(qa) + p.dlo);
    const long hi = (p.dhi >= kNoBound) ? klast : lmin_(klast, static_cast<long>(qa) + p.dhi);
    return lo > hi;
  };
  if (row_empty(qa0) || row_empty(qa1)) {
    s.lo = 0; s.hi = n_kv_tiles - 1;  // reference semantics: iterate every key
    return s;
  }
  long jlo = (p.dlo <= -kNoBound) ? 0 : static_cast<long>(qa0) + p.dlo - p.k_off;
  long jhi = (p.dhi >= kNoBound) ? p.n_kv - 1 : static_cast<long>(qa1) + p.dhi - p.k_off;
  jlo = lmax_(jlo, 0L);
  jhi = lmin_(jhi, static_cast<long>(p.n_kv - 1));
  s.lo = static_cast<int>(jlo / BN);
  s.hi = static_cast<int>(jhi / BN);
  return s;
}

// A work unit: one KV head g of sequence b and one pair of query slots (two
// heads of the group, or two query tiles of a one-head group). Its key tiles
// are the union [J0, J1] of both slots'.
struct Unit {
  SlotInfo sl[2];
  bool act1;
  int b, g, J0, J1, len;
};

__host__ __device__ inline Unit unit_info(const Params& p, int u) {
  Unit U;
  U.g = u % p.n_kv_heads;
  const int t = u / p.n_kv_heads;
  U.b = t % p.batch;
  // One-unit-per-CTA mode: heaviest first, for the hardware's greedy CTA
  // scheduling. Split mode: heavy and light pairs alternate, so no CTA's
  // range collects a long run of short units (each costs a Q load and an
  // epilogue).
  const int tb = t / p.batch;
  const int pair = !p.split ? p.pairs_per_group - 1 - tb
                            : ((tb & 1) ? tb / 2 : p.pairs_per_group - 1 - tb / 2);
  U.sl[0] = slot_info(p, U.g, 2 * pair);
  U.sl[1] = slot_info(p, U.g, 2 * pair + 1);
  const bool act0 = U.sl[0].lo <= U.sl[0].hi;
  U.act1 = U.sl[1].lo <= U.sl[1].hi;
  if (!act0 && !U.act1) { U.J0 = 0; U.J1 = -1; }
  else if (!U.act1) { U.J0 = U.sl[0].lo; U.J1 = U.sl[0].hi; }
  else if (!act0) { U.J0 = U.sl[1].lo; U.J1 = U.sl[1].hi; }
  else {
    U.J0 = U.sl[0].lo < U.sl[1].lo ? U.sl[0].lo : U.sl[1].lo;
    U.J1 = U.sl[0].hi > U.sl[1].hi ? U.sl[0].hi : U.sl[1].hi;
  }
  U.len = U.J1 - U.J0 + 1;
  return U;
}

// Split mode works in "cost" positions: a unit with len > 0 key tiles costs
// item_cost + len positions, the first item_cost standing for the per-item
// overhead (Q load, pipeline refill, epilogue) and tile t at position
// pre + item_cost + t. CTA c owns positions [c*W/G, (c+1)*W/G), so CTAs
// that meet many short units get fewer tiles.
__host__ __device__ __forceinline__ int split_begin(const Params& p, int c) {
  return static_cast<int>(static_cast<long long>(c) * p.W / p.G);
}
__device__ __forceinline__ int split_cta(const Params& p, long long x) {
  return static_cast<int>(((x + 1) * p.G - 1) / p.W);
}

// One CTA's walk over its items: a contiguous key-tile range [ja, jb] of one
// unit. Every warp role walks the same sequence.
struct Item {
  Unit U;
  int u, pre;    // unit index and its first cost position
  int ja, jb;    // key tiles of this item
  bool full;     // the item is the whole unit (no partial results)
  bool first;    // first item of this CTA
};

struct Walk {
  int u, pre, pos, end, k;
  template <bool SPLIT>
  __device__ __forceinline__ void begin(const Params& p, const SplitPlan& plan) {
    k = 0;
    if (SPLIT) {
      pos = split_begin(p, blockIdx.x);
      end = split_begin(p, blockIdx.x + 1);
      u = plan.u0[blockIdx.x];
      pre = plan.pre0[blockIdx.x];
    } else {
      u = blockIdx.x;
      pre = 0;
      pos = 0;
      end = -1;  // one whole unit
    }
  }
  template <bool SPLIT>
  __device__ __forceinline__ bool next(const Params& p, Item& it) {
    if (!SPLIT) {
      if (end == 0 || u >= p.n_units) return false;
      end = 0;
      it.U = unit_info(p, u);
      if (it.U.len <= 0) return false;
      it.u = u;
      it.pre = 0;
      it.ja = it.U.J0;
      it.jb = it.U.J1;
      it.full = true;
      it.first = true;
      ++k;
      return true;
    }
    for (;;) {
      if (pos >= end || u >= p.n_units) return false;
      it.U = unit_info(p, u);
      if (it.U.len <= 0) {  // no keys: costs nothing
        ++u;
        continue;
      }
      const int base = pre + p.item_cost;  // cost position of tile 0
      const int t0 = pos > base ? pos - base : 0;
      const int t1 = (end - base < it.U.len) ? end - base : it.U.len;
      const int cost = p.item_cost + it.U.len;
      const int upre = pre, uu = u;
      if (end >= pre + cost) {  // the unit ends inside this CTA's range
        pos = pre + cost;
        pre += cost;
        ++u;
      } else {
        pos = end;
      }
      if (t1 <= t0) continue;  // only the unit's overhead positions fall here
      it.u = uu;
      it.pre = upre;
      it.ja = it.U.J0 + t0;
      it.jb = it.U.J0 + t1 - 1;
      it.full = t0 == 0 && t1 == it.U.len;
      it.first = k == 0;
      ++k;
      return true;
    }
  }
};

// Partial results of a split unit: per CTA two records (its first and its
// last item), per slot the unnormalised O as [D/4][BM] float4 (a warp's 32
// rows of one column quad are 512 contiguous bytes), then m[BM] and l[BM].
template <int D>
__device__ __forceinline__ float* record(const Params& p, int cta, int r, int s) {
  constexpr int REC = BM * D + 2 * BM;
  return p.rec + (static_cast<size_t>(cta) * 4 + r * 2 + s) * REC;
}

// SPLIT: the split schedule (Params::split != 0); the one-CTA-per-unit
// instantiation compiles without the multi-item walk and partial records.
template <int D, bool BF16, bool SOFTCAP, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmQt,
            const __grid_constant__ CUtensorMap tmKt, const __grid_constant__ CUtensorMap tmVt,
            Params p, const __grid_constant__ SplitPlan plan) {
  using L = Smem<D>;
  constexpr int KS = L::K_STAGES, VS = L::V_STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars;                      // [1]
  uint64_t* q_empty = q_full + 1;               // [1]
  uint64_t* k_full = q_empty + 1;               // [KS]
  uint64_t* k_empty = k_full + KS;              // [KS]
  uint64_t* v_full = k_empty + KS;              // [VS]
  uint64_t* v_empty = v_full + VS;              // [VS]
  uint64_t* s_full = v_empty + VS;              // [slot] S of the slot's next tile is in TMEM
  uint64_t* p_full = s_full + 2;                // [slot] P is in TMEM (4 softmax warps)
  uint64_t* o_done = p_full + 2;                // [slot] a P·V retired
  uint64_t* o_free = o_done + 2;                // [slot] the item's O was read out
  uint64_t* pub_bar = o_free + 2;               // [slot] a split part's record is written
  uint64_t* dec_bar = pub_bar + 2;              // [slot] the last-arriver decision is made
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dec_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);  // [slot]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_free[i], 4);
      mbar_init(&pub_bar[i], 4);
      mbar_init(&dec_bar[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  Walk w;
  w.begin<SPLIT>(p, plan);
  Item item;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    if (elect_one_sync()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      // Column `col` of head `head`, rows from `row`: a 2-D map over the
      // rows' head-major columns, or a [rows, heads, d_out] view.
      const bool h3 = p.head3d != 0;
      auto load = [h3](void* dst, const CUtensorMap* map, uint64_t* bar, int head, int col, int row) {
        if (h3) tma_load_3d(dst, map, bar, col, head, row);
        else tma_load_2d(dst, map, bar, head * D + col, row);
      };
      int kv_base = 0;  // ring position of the item's first tile, continued across items
      bool ok = true;
      for (int k = 0; ok && w.template next<SPLIT>(p, item); ++k) {
        const Unit& U = item.U;
        const int q_row0 = U.b * p.n_q, kv_row0 = U.b * p.n_kv;
        // The Q buffers are reused once every S of the previous item retired.
        if (k > 0 && !mbar_wait(q_empty, (k - 1) & 1, p.err, abort_flag)) break;
        const int nslots = U.act1 ? 2 : 1;
        mbar_arrive_expect_tx(q_full, nslots * L::Q_TILE);
        for (int s = 0; s < nslots; ++s) {
          for (int a = 0; a < L::ATOMS; ++a)
            load(smem + L::Q_OFF + s * L::Q_TILE + a * L::Q_ATOM, &tmQ, q_full, U.sl[s].head, a * 64,
                 q_row0 + U.sl[s].qt * BM);
          if (L::TAIL)
            load(smem + L::Q_OFF + s * L::Q_TILE + L::Q_TAIL_OFF, &tmQt, q_full, U.sl[s].head, L::ATOMS * 64,
                 q_row0 + U.sl[s].qt * BM);
        }
        // K tile j at ring position kv_base + j - ja of the K ring, V tile j
        // at the same position of the V ring.
        auto load_kv = [&](bool is_k, int j) -> bool {
          const int pos = kv_base + j - item.ja;
          const int nst = is_k ? KS : VS;
          const int st = pos % nst;
          const uint32_t ph = ((pos / nst) & 1) ^ 1;
          uint64_t* empty = is_k ? &k_empty[st] : &v_empty[st];
          uint64_t* full = is_k ? &k_full[st] : &v_full[st];
          if (!mbar_wait(empty, ph, p.err, abort_flag)) return false;
          mbar_arrive_expect_tx(full, L::KV_TILE);
          uint8_t* dst = smem + (is_k ? L::K_OFF : L::V_OFF) + st * L::KV_TILE;
          const CUtensorMap* map = is_k ? &tmK : &tmV;
          for (int a = 0; a < L::ATOMS; ++a)
            load(dst + a * L::KV_ATOM, map, full, U.g, a * 64, kv_row0 + j * BN);
          if (L::TAIL)
            load(dst + L::KV_TAIL_OFF, is_k ? &tmKt : &tmVt, full, U.g, L::ATOMS * 64, kv_row0 + j * BN);
          return true;
        };
        // K runs one tile ahead of V: the UMMA warp issues S(j+1) right
        // behind P·V(j).
        ok = load_kv(true, item.ja);
        for (int j = item.ja; ok && j <= item.jb; ++j) {
          if (j + 1 <= item.jb && !(ok = load_kv(true, j + 1))) break;
          ok = load_kv(false, j);
        }
        kv_base += item.jb - item.ja + 1;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = idesc_f16(BM, BN, BF16, false, false);
      constexpr uint32_t idesc_o = idesc_f16(BM, L::ATOMS * 64, BF16, false, true);
      constexpr uint32_t idesc_ot = idesc_f16(BM, L::TAIL ? L::TAIL : 16, BF16, false, true);
      const uint32_t q_addr = smem_u32(smem + L::Q_OFF);
      const uint32_t k_addr = smem_u32(smem + L::K_OFF);
      const uint32_t v_addr = smem_u32(smem + L::V_OFF);
      // Base descriptors; each UMMA advances them by a constant byte offset.
      const uint64_t q_desc = desc_kmajor_sw128(q_addr), k_desc = desc_kmajor_sw128(k_addr);
      const uint64_t v_desc = desc_mnmajor_sw128(v_addr, L::KV_ATOM, 1024);
      const uint64_t qt_desc = desc_kmajor_sw32(q_addr), kt_desc = desc_kmajor_sw32(k_addr);
      const uint64_t vt_desc = desc_mnmajor_sw32(v_addr);
      int n_pv[2] = {0, 0};   // P·V issued per slot (all items)
      int n_out[2] = {0, 0};  // items whose O the slot's softmax warps have taken out
      int kv_base = 0;        // ring position of the item's first tile
      bool ok = true;
      for (int k = 0; ok && w.template next<SPLIT>(p, item); ++k) {
        int rlo[2], rhi[2];
        for (int s = 0; s < 2; ++s) {
          const bool act = s == 0 || item.U.act1;
          rlo[s] = act ? max(item.ja, item.U.sl[s].lo) : 1;
          rhi[s] = act ? min(item.jb, item.U.sl[s].hi) : 0;
        }
        bool first_pv[2] = {true, true};
        ok = mbar_wait(q_full, k & 1, p.err, abort_flag);
        auto pos_of = [&](int j) { return kv_base + j - item.ja; };
        // S = Q K_j^T of slot s into the slot's S columns. They last held
        // P(j-1), read by this slot's P·V(j-1), which this thread issued
        // earlier: UMMAs issued by one thread execute in issue order, so the
        // overwrite needs no wait.
        auto issue_s = [&](int j, int s) {
          const uint32_t st = pos_of(j) % KS;
          const uint32_t d_tmem = tmem_base + s * 256;
#pragma unroll
          for (int ks = 0; ks < L::ATOMS * 4; ++ks) {
            const uint32_t qo = (ks >> 2) * L::Q_ATOM + (ks & 3) * 32;
            const uint32_t ko = (ks >> 2) * L::KV_ATOM + (ks & 3) * 32;
            umma_f16_ss(d_tmem, desc_add(q_desc, s * L::Q_TILE + qo),
                        desc_add(k_desc, st * L::KV_TILE + ko), idesc_s, ks > 0);
          }
          if (L::TAIL) {  // the 16-column tail: one K step on 32-B-swizzled rows
            umma_f16_ss(d_tmem, desc_add(qt_desc, s * L::Q_TILE + L::Q_TAIL_OFF),
                        desc_add(kt_desc, st * L::KV_TILE + L::KV_TAIL_OFF), idesc_s, 1u);
          }
          umma_commit(&s_full[s]);
        };
        int k_ready = item.ja - 1;  // last key tile whose K load has been awaited
        auto wait_k = [&](int j) -> bool {
          if (j <= k_ready) return true;
          if (!mbar_wait(&k_full[pos_of(j) % KS], (pos_of(j) / KS) & 1, p.err, abort_flag)) return false;
          tc_fence_after();
          k_ready = j;
          return true;
        };
        for (int j = item.ja; ok && j <= item.jb; ++j) {
          // S(j) of the slots whose range starts at tile j (the others' S(j)
          // went out behind their P·V(j-1)).
          for (int s = 0; ok && s < 2; ++s)
            if (rlo[s] <= rhi[s] && rlo[s] == j && (ok = wait_k(j))) issue_s(j, s);
          // Every S that reads K tile j is issued: hand its stage back (the
          // load is awaited first even when no slot reads the tile), and Q
          // after the item's last tile.
          if (!ok || !(ok = wait_k(j))) break;
          umma_commit(&k_empty[pos_of(j) % KS]);
          if (j == item.jb) umma_commit(q_empty);
          // Per slot, in ping-pong order: O += P_j V_j as soon as the slot's
          // P is in TMEM, then the slot's S(j+1).
          const uint32_t vs = pos_of(j) % VS;
          bool v_ready = false;
          for (int s = 0; ok && s < 2; ++s) {
            if (!(rlo[s] <= j && j <= rhi[s])) continue;
            if (!(ok = mbar_wait(&p_full[s], n_pv[s] & 1, p.err, abort_flag))) break;
            tc_fence_after();
            if (first_pv[s] && n_out[s] > 0) {
              // O is overwritten: the previous item's O must have been read out.
              if (!(ok = mbar_wait(&o_free[s], (n_out[s] - 1) & 1, p.err, abort_flag))) break;
              tc_fence_after();
            }
            if (!v_ready) {
              if (!(ok = mbar_wait(&v_full[vs], (pos_of(j) / VS) & 1, p.err, abort_flag))) break;
              tc_fence_after();
              v_ready = true;
            }
            const uint32_t o_tmem = tmem_base + s * 256 + 128;
            const uint32_t p_tmem = tmem_base + s * 256;
#pragma unroll
            for (int ks = 0; ks < BN / 16; ++ks) {
              const uint32_t acc = (!first_pv[s] || ks > 0) ? 1u : 0u;
              const uint64_t vd = desc_add(v_desc, vs * L::KV_TILE + ks * 2048);
              umma_f16_ts(o_tmem, p_tmem + ks * 8, vd, idesc_o, acc);
              if (L::TAIL) {  // O columns [64*ATOMS, D) from the tail atom (16 key rows = 512 B)
                const uint64_t vt = desc_add(vt_desc, vs * L::KV_TILE + L::KV_TAIL_OFF + ks * 512);
                umma_f16_ts(o_tmem + L::ATOMS * 64, p_tmem + ks * 8, vt, idesc_ot, acc);
              }
            }
            umma_commit(&o_done[s]);
            ++n_pv[s];
            first_pv[s] = false;
            if (j + 1 <= rhi[s] && (ok = wait_k(j + 1))) issue_s(j + 1, s);
          }
          if (!ok) break;
          // A tile neither slot reads still has its load awaited before the
          // stage is handed back.
          if (!v_ready && !(ok = mbar_wait(&v_full[vs], (pos_of(j) / VS) & 1, p.err, abort_flag))) break;
          umma_commit(&v_empty[vs]);
        }
        for (int s = 0; s < 2; ++s)
          if (rlo[s] <= rhi[s]) ++n_out[s];
        kv_base += item.jb - item.ja + 1;
      }
    }
  } else if (warp >= kSoftWarp0) {
    // ------------------------------------------------------------ softmax
    const int s = (warp - kSoftWarp0) >> 2;
    const int quarter = warp & 3;  // TMEM lanes 32*(warp % 4): each slot's four warps cover all 128
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t s_col = s * 256;
    const uint32_t o_col = s * 256 + 128;
    int it = 0;      // tiles this slot has processed (all items): barrier phases
    int n_part = 0;  // split parts this slot has published
    bool ok = true;
    while (ok && w.template next<SPLIT>(p, item)) {
      const Unit& U = item.U;
      if (s == 1 && !U.act1) continue;
      const SlotInfo me = s == 0 ? U.sl[0] : U.sl[1];  // no runtime index into sl[]
      const int lo = max(item.ja, me.lo), hi = min(item.jb, me.hi);
      const int qa = p.q_off + me.qt * BM + row;  // absolute query position
      const int qa_min = p.q_off + me.qt * BM, qa_max = qa_min + BM - 1;
      float m_used = -INFINITY, l = 0.0f;
      for (int j = lo; j <= hi; ++j, ++it) {
        const bool first_tile = j == lo;
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[s], it & 1, p.err, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        float x[BN];
        {
          uint32_t r0[32], r1[32], r2[32], r3[32];
          tmem_ld32(lane_base + s_col, r0);
          tmem_ld32(lane_base + s_col + 32, r1);
          tmem_ld32(lane_base + s_col + 64, r2);
          tmem_ld32(lane_base + s_col + 96, r3);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            x[i] = __uint_as_float(r0[i]);
            x[32 + i] = __uint_as_float(r1[i]);
            x[64 + i] = __uint_as_float(r2[i]);
            x[96 + i] = __uint_as_float(r3[i]);
          }
        }
        if (SOFTCAP) {
          // s = softcap * tanh(s*scale / softcap), then back to "raw" units so
          // the common scaling below applies.
#pragma unroll
          for (int i = 0; i < BN; ++i) {
            const float v = __fmul_rn(x[i], p.scale);
            x[i] = p.softcap * tanhf(v / p.softcap) / p.scale;
          }
        }
        const int ka0 = p.k_off + j * BN;  // absolute key of column 0
        const int kvalid = p.n_kv - j * BN;
        const bool interior = (kvalid >= BN) &&
            (p.dlo <= -kNoBound || ka0 - qa_max >= p.dlo) &&
            (p.dhi >= kNoBound || ka0 + BN - 1 - qa_min <= p.dhi);
        // This row's visible keys in the tile: the band's interval [vlo, vhi]
        // cut to the real keys [0, rlast] (everything on interior tiles).
        const int rlast = (kvalid < BN ? kvalid : BN) - 1;
        int vlo = 0, vhi = BN - 1;
        if (!interior) {
          const long a = static_cast<long>(qa) + p.dlo - ka0, b = static_cast<long>(qa) + p.dhi - ka0;
          vlo = p.dlo <= -kNoBound ? 0 : static_cast<int>(a < 0 ? 0 : (a > BN ? BN : a));
          vhi = p.dhi >= kNoBound ? rlast : static_cast<int>(b > rlast ? rlast : (b < -1 ? -1 : b));
        }
        // Tile max in log2 units: max over visible of s*c, floored at the clamp
        // (masked real keys score exactly the clamp).
        float mraw;
        if (interior) {
          float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
          for (int i = 0; i < BN; i += 8) {
            m0 = max3(m0, x[i], x[i + 1]);
            m1 = max3(m1, x[i + 2], x[i + 3]);
            m2 = max3(m2, x[i + 4], x[i + 5]);
            m3 = max3(m3, x[i + 6], x[i + 7]);
          }
          mraw = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
        } else {
          mraw = -INFINITY;
#pragma unroll
          for (int i = 0; i < BN; ++i) mraw = fmaxf(mraw, (i >= vlo && i <= vhi) ? x[i] : -INFINITY);
        }
        const float mt = fmaxf(mraw * p.scale_log2, kClamp2);
        // Lazy rescale of the exponent base.
        float alpha = 1.0f;
        bool need = false;
        if (first_tile) {
          m_used = mt;
        } else if (mt > m_used + kRescaleThresh) {
          alpha = fast_exp2(m_used - mt);
          m_used = mt;
          need = true;
        }
        const bool fast = __all_sync(0xffffffffu, m_used >= kClamp2 + kFastMargin);
        const float c = p.scale_log2, nm = -m_used;
        uint64_t rs[2] = {0ull, 0ull};  // packed row-sum partials (+0.0f pairs)
        // P over the first BN/2 columns of S, 32 keys (16 columns) at a time.
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t pk[16];
          if (fast && interior) {  // the common case: no mask, no clamp
            const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(nm, nm);
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float y0, y1, p0, p1;
              f2_unpack(f2_fma(f2_pack(x[c0 + i], x[c0 + i + 1]), c2, nm2), y0, y1);
              if (poly_every<D>() > 0 && (i / 2) % poly_every<D>() == poly_every<D>() - 1) {
                exp2_poly2(y0, y1, p0, p1);
              } else {
                p0 = fast_exp2(y0);
                p1 = fast_exp2(y1);
              }
              rs[(i / 2) & 1] = f2_add(rs[(i / 2) & 1], f2_pack(p0, p1));
              pk[i / 2] = pack2<BF16>(p0, p1);
            }
          } else if (fast) {
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const int k0 = c0 + i;
              float p0 = fast_exp2(fmaf(x[k0], c, nm));
              float p1 = fast_exp2(fmaf(x[k0 + 1], c, nm));
              p0 = (k0 >= vlo && k0 <= vhi) ? p0 : 0.0f;
              p1 = (k0 + 1 >= vlo && k0 + 1 <= vhi) ? p1 : 0.0f;
              rs[(i / 2) & 1] = f2_add(rs[(i / 2) & 1], f2_pack(p0, p1));
              pk[i / 2] = pack2<BF16>(p0, p1);
            }
          } else {
            // Exact path near the clamp: y = visible ? max(s*c, clamp) :
            // (real key ? clamp : -inf).
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const int k0 = c0 + i;
              float y0 = fmaxf(x[k0] * c, kClamp2), y1 = fmaxf(x[k0 + 1] * c, kClamp2);
              if (!(k0 >= vlo && k0 <= vhi)) y0 = k0 <= rlast ? kClamp2 : -INFINITY;
              if (!(k0 + 1 >= vlo && k0 + 1 <= vhi)) y1 = k0 + 1 <= rlast ? kClamp2 : -INFINITY;
              const float p0 = fast_exp2(y0 + nm), p1 = fast_exp2(y1 + nm);
              rs[(i / 2) & 1] = f2_add(rs[(i / 2) & 1], f2_pack(p0, p1));
              pk[i / 2] = pack2<BF16>(p0, p1);
            }
          }
          tmem_st16(lane_base + s_col + c0 / 2, pk);
        }
        float rs0, rs1, rs2, rs3;
        f2_unpack(rs[0], rs0, rs1);
        f2_unpack(rs[1], rs2, rs3);
        l = l * alpha + ((rs0 + rs1) + (rs2 + rs3));
        // O is idle here: this slot's S(j) was issued behind its P·V(j-1),
        // so S(j)'s commit retired it, and P·V(j) waits for p_full.
        if (__any_sync(0xffffffffu, need)) {
          uint32_t r[32];
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 32) {
            tmem_ld32(lane_base + o_col + c0, r);
            tmem_wait_ld();
            uint32_t lo16[16], hi16[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              lo16[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
              hi16[i] = __float_as_uint(__uint_as_float(r[16 + i]) * alpha);
            }
            tmem_st16(lane_base + o_col + c0, lo16);
            tmem_st16(lane_base + o_col + c0 + 16, hi16);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[s]);
      }
      if (!ok) break;
      const bool has = lo <= hi;
      // Wait for the item's last P·V.
      if (has) {
        if (!__all_sync(0xffffffffu, mbar_wait(&o_done[s], (it - 1) & 1, p.err, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      const int qrow = me.qt * BM + row;
      uint16_t* out_row = reinterpret_cast<uint16_t*>(p.out) +
                          static_cast<int64_t>(U.b * p.n_q + qrow) * p.ldo + me.head * p.d_out;
      // Normalised store of one 32-column chunk.
      auto store_chunk = [&](int c0, const float (&v)[32], float inv_l) {
        if (qrow >= p.n_q) return;
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack2<BF16>(v[2 * i] * inv_l, v[2 * i + 1] * inv_l);
        uint4* dst = reinterpret_cast<uint4*>(out_row + c0);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (c0 + 8 * i + 8 <= p.d_out)  // 8-column groups of the real head width
            dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      };
      if (!SPLIT || item.full) {
        // All of O's columns in one batch of TMEM loads (one load latency).
        const float inv_l = 1.0f / l;
        constexpr int NCH = (D + 31) / 32;
        uint32_t r[NCH][32];
#pragma unroll
        for (int c = 0; c < NCH; ++c) tmem_ld32(lane_base + o_col + c * 32, r[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[c][i]);
          store_chunk(c * 32, v, inv_l);
        }
      } else {
        // Part of a unit split over CTAs c_first..c_last: publish (O, m, l);
        // the last part to arrive merges every part's record in CTA order.
        const long long tpos = static_cast<long long>(item.pre) + p.item_cost;  // tile 0's position
        const int c_first = split_cta(p, tpos), c_last = split_cta(p, tpos + U.len - 1);
        float* rec = record<D>(p, blockIdx.x, item.first ? 0 : 1, s);
        if (has) {
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(lane_base + o_col + c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int q4 = c0 / 4 + i;
              if (4 * q4 + 4 <= D)
                __stcg(reinterpret_cast<float4*>(rec) + q4 * BM + row,
                       make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                   __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])));
            }
          }
        }
        __stcg(rec + BM * D + row, has ? m_used : -INFINITY);
        __stcg(rec + BM * D + BM + row, has ? l : 0.0f);
        __threadfence();
        // The slot's four warps have published; one thread counts the part in.
        __syncwarp();
        if (lane == 0) mbar_arrive(&pub_bar[s]);
        if (row == 0) {
          bool okp = mbar_wait(&pub_bar[s], n_part & 1, p.err, abort_flag);
          int last = 0;
          if (okp) {
            int* cnt = p.cnt + 2 * item.u + s;
            const int parts = c_last - c_first + 1;
            const int old = atomicAdd(cnt, 1);
            last = old == parts - 1;
            if (last) atomicExch(cnt, 0);  // ready for the next launch
          }
          last_flag[s] = last;
          mbar_arrive(&dec_bar[s]);
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&dec_bar[s], n_part & 1, p.err, abort_flag))) {
          ok = false;
          break;
        }
        ++n_part;
        if (last_flag[s]) {
          __threadfence();
          // One pass over the parts in CTA order with a running max (the
          // result does not depend on which part arrived last), GC columns
          // at a time.
          constexpr int GC = (D % 64 == 0) ? 64 : 32;
#pragma unroll 1
          for (int g0 = 0; g0 < D; g0 += GC) {
            float acc[GC];
#pragma unroll
            for (int i = 0; i < GC; ++i) acc[i] = 0.0f;
            float M = -INFINITY, Lsum = 0.0f;
            for (int cc = c_first; cc <= c_last; ++cc) {
              // u is CTA cc's first item unless an earlier unit's tiles precede it there
              const int rr = (cc == c_first && split_begin(p, cc) < item.pre) ? 1 : 0;
              const float* rc = record<D>(p, cc, rr, s);
              const float mc = __ldcg(rc + BM * D + row), lc = __ldcg(rc + BM * D + BM + row);
              float v[GC];
              if (cc == static_cast<int>(blockIdx.x)) {  // this CTA's part: still in TMEM
                if (!has) continue;
#pragma unroll
                for (int h = 0; h < GC; h += 32) {
                  uint32_t r[32];
                  tmem_ld32(lane_base + o_col + g0 + h, r);
                  tmem_wait_ld();
#pragma unroll
                  for (int i = 0; i < 32; ++i) v[h + i] = __uint_as_float(r[i]);
                }
              } else {
                const float4* src = reinterpret_cast<const float4*>(rc) + (g0 / 4) * BM + row;
#pragma unroll
                for (int i = 0; i < GC / 4; ++i) {
                  float4 v4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                  if (g0 + 4 * i + 4 <= D) v4 = __ldcg(src + i * BM);
                  v[4 * i] = v4.x;
                  v[4 * i + 1] = v4.y;
                  v[4 * i + 2] = v4.z;
                  v[4 * i + 3] = v4.w;
                }
              }
              if (!(lc > 0.0f)) continue;  // a part without keys for this slot
              const float Mn = fmaxf(M, mc);
              const float a = fast_exp2(M - Mn), wc = fast_exp2(mc - Mn);
#pragma unroll
              for (int i = 0; i < GC; ++i) acc[i] = fmaf(wc, v[i], acc[i] * a);
              Lsum = fmaf(wc, lc, Lsum * a);
              M = Mn;
            }
            const float inv_l = 1.0f / Lsum;
#pragma unroll
            for (int h = 0; h < GC; h += 32) {
              float o32[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) o32[i] = acc[h + i];
              if (g0 + h < D) store_chunk(g0 + h, o32, inv_l);
            }
          }
        }
      }
      if (has) {  // O has been read: the next item's first P·V may overwrite it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[s]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_after_abort();  // let in-flight TMA / UMMA work retire
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <int D, bool BF16, bool SOFTCAP, bool SPLIT>
static int launch_impl(const CUtensorMap* tm, const Params& p, const SplitPlan& plan, dim3 grid,
                       cudaStream_t stream) {
  static uint64_t configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    if (cudaFuncSetAttribute(attn_kernel<D, BF16, SOFTCAP, SPLIT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, Smem<D>::BYTES) != cudaSuccess)
      return RB_E_DEVICE;
    configured |= 1ull << (dev & 63);
  }
  attn_kernel<D, BF16, SOFTCAP, SPLIT><<<grid, kThreads, Smem<D>::BYTES, stream>>>(tm[0], tm[1], tm[2], tm[3],
                                                                          tm[4], tm[5], p, plan);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return report_error(RB_E_DEVICE, cudaGetErrorString(e));
  return RB_OK;
}

template <int D, bool SPLIT>
static int launch_s(const CUtensorMap* tm, const Params& p, const SplitPlan& plan, dim3 grid, bool bf16,
                    cudaStream_t stream) {
  if (p.softcap != 0.0f)
    return bf16 ? launch_impl<D, true, true, SPLIT>(tm, p, plan, grid, stream)
                : launch_impl<D, false, true, SPLIT>(tm, p, plan, grid, stream);
  return bf16 ? launch_impl<D, true, false, SPLIT>(tm, p, plan, grid, stream)
              : launch_impl<D, false, false, SPLIT>(tm, p, plan, grid, stream);
}

template <int D>
static int launch_d(const CUtensorMap* tm, const Params& p, const SplitPlan& plan, dim3 grid, bool bf16,
                    cudaStream_t stream) {
  return p.split ? launch_s<D, true>(tm, p, plan, grid, bf16, stream)
                 : launch_s<D, false>(tm, p, plan, grid, bf16, stream);
}

}  // namespace attn

int set_attention_split(int policy) { return attn::g_split_policy.exchange(policy); }

int launch_attention(const CUtensorMap* tm, const AttnLaunch& L, cudaStream_t stream) {
  using namespace attn;
  Params p{};
  p.out = L.out;
  p.n_q = L.n_q;
  p.n_kv = L.n_kv;
  p.n_head = L.n_head;
  p.n_kv_heads = L.n_kv_heads;
  p.group = L.n_head / L.n_kv_heads;
  p.ldo = L.ldo;
  p.q_tiles = (L.n_q + BM - 1) / BM;
  p.pairs_per_group = (p.group * p.q_tiles + 1) / 2;
  p.scale = L.scale;
  p.scale_log2 = L.scale * kLog2e;
  p.softcap = L.softcap;
  p.err = L.err;
  p.d_out = L.d_out;
  p.head3d = L.head_maps;
  p.batch = L.batch > 0 ? L.batch : 1;
  // Mask band in relative coordinates (key - query).
  auto clampw = [](int64_t w) { return static_cast<int>(w > (kNoBound / 2) ? (kNoBound / 2) : w); };
  p.dlo = -kNoBound;
  p.dhi = kNoBound;
  p.q_off = 0;
  p.k_off = 0;
  switch (L.mask_mode) {
    case RB_MASK_NONE:
    case RB_MASK_NONE_BLOCK:
      break;
    case RB_MASK_CAUSAL:
      p.dhi = 0;
      break;
    case RB_MASK_WINDOW:
      p.dlo = -clampw(L.window);
      p.dhi = clampw(L.window);
      break;
    case RB_MASK_CAUSAL_WINDOW:
      p.dlo = 1 - clampw(L.window);
      p.dhi = 0;
      break;
    case RB_MASK_WINDOW_BLOCK:
      p.dlo = -clampw(L.window);
      p.dhi = clampw(L.window);
      p.q_off = static_cast<int>(L.q_start);
      p.k_off = static_cast<int>(L.kv_start);
      break;
    case RB_MASK_CAUSAL_BLOCK:
      if (L.window >= 0) p.dlo = 1 - clampw(L.window);
      p.dhi = 0;
      p.q_off = static_cast<int>(L.q_start);
      p.k_off = static_cast<int>(L.kv_start);
      break;
    default:
      return RB_E_SHAPE;
  }
  const long long units = static_cast<long long>(p.pairs_per_group) * L.n_kv_heads * p.batch;
  if (units <= 0 || units > (1ll << 30)) return RB_E_SHAPE;
  p.n_units = static_cast<int>(units);
  p.split = 0;
  // Split mode: the units' key tiles, concatenated, are cut into G equal
  // ranges, one per SM, so the last wave does not leave SMs idle; a unit cut
  // by a range boundary is finished by whichever of its parts arrives last.
  // A unit's length depends only on its slot pair (not on KV head or
  // sequence): units come in blocks of batch * n_kv_heads of one length.
  SplitPlan plan{};
  const int policy = g_split_policy.load();
  if (policy != RB_ATTN_SPLIT_NEVER && L.ws_rec && L.ws_cnt && units <= kAttnMaxUnits && L.num_sms > 0) {
    // A unit's length depends only on its slot pair (not on KV head or
    // sequence): units come in blocks of batch * n_kv_heads of one pair.
    const int blk = p.batch * L.n_kv_heads;
    const int P = p.pairs_per_group;
    std::vector<int> plen(P);  // key tiles of the units of slot pair `pair`
    for (int pair = 0; pair < P; ++pair) {
      p.split = 0;  // one-CTA-per-unit order: block t holds pair P-1-t
      plen[pair] = std::max(0, unit_info(p, (P - 1 - pair) * blk).len);
    }
    p.split = 1;  // split-mode order (heavy and light pairs alternate)
    std::vector<long long> bcost(P), bpre(P);
    long long W = 0;
    for (int t = 0; t < P; ++t) {
      const int pair = (t & 1) ? t / 2 : P - 1 - t / 2;
      bcost[t] = plen[pair] > 0 ? kItemCost + plen[pair] : 0;  // per unit of block t
      bpre[t] = W;
      W += blk * bcost[t];
    }
    const int G = static_cast<int>(std::min<long long>(W, std::min(L.num_sms, kMaxCtas)));
    bool use = W > 0 && W < (1ll << 30);
    if (use && policy == RB_ATTN_SPLIT_AUTO) {
      // Estimated finish time, in key tiles, of the one-CTA-per-unit greedy
      // schedule (heaviest first onto the first free SM) against the split.
      long long tiles = 0;
      bool equal = true;  // every unit has the same length (no causal / window mask)
      for (int pair = 0; pair < P; ++pair) {
        tiles += static_cast<long long>(blk) * plen[pair];
        equal = equal && plen[pair] == plen[0];
      }
      const double split_t = (static_cast<double>(tiles) + kItemTime * static_cast<double>(units)) / G + kMergeTime;
      if (units <= 4 * 65536) {
        std::priority_queue<long long, std::vector<long long>, std::greater<long long>> sm;
        for (int i = 0; i < L.num_sms; ++i) sm.push(0);
        for (int pair = P - 1; pair >= 0; --pair)
          for (int i = 0; i < blk; ++i) {
            const long long t0 = sm.top();
            sm.pop();
            sm.push(t0 + plen[pair] + static_cast<long long>(kCtaTime));
          }
        long long greedy = 0;
        while (!sm.empty()) {
          greedy = std::max(greedy, sm.top());
          sm.pop();
        }
        // Units of unequal length leave the split's shares uneven in time
        // (short items cost more than modelled): it must win clearly there.
        // Equal units: measured on config #4's tower (2560 units of 38 key
        // tiles, head_dim 72), the split estimated at 0.94 of the greedy
        // finish ran 2.5-5% slower, its records and merges costing more than
        // modelled; config #3's forward (2048 units of 8 key tiles, 0.93) ran
        // as fast either way; config #2's bidirectional call (0.81) gains from
        // it. So it must beat the greedy estimate by 10%.
        use = split_t < (equal ? 0.90 : 0.75) * static_cast<double>(greedy);
      } else {
        use = false;  // many units: the greedy schedule's last wave is short
      }
    }
    p.split = 0;
    if (use) {
      p.split = 1;
      p.W = static_cast<int>(W);
      p.G = G;
      p.item_cost = kItemCost;
      p.rec = L.ws_rec;
      p.cnt = L.ws_cnt;
      int t = 0;
      for (int c = 0; c < G; ++c) {
        const long long b0 = static_cast<long long>(c) * W / G;
        while (t + 1 < P && bpre[t] + blk * bcost[t] <= b0) ++t;
        const long long i = (b0 - bpre[t]) / bcost[t];  // bcost[t] > 0: position b0 lies in block t
        plan.u0[c] = static_cast<int>(t * blk + i);
        plan.pre0[c] = static_cast<int>(bpre[t] + i * bcost[t]);
      }
    }
  }
  const dim3 grid(p.split ? p.G : p.n_units);
  const bool bf16 = L.dtype == RB_DTYPE_BF16;
  if (L.head_dim == 128) return launch_d<128>(tm, p, plan, grid, bf16, stream);
  if (L.head_dim == 64) return launch_d<64>(tm, p, plan, grid, bf16, stream);
  if (L.head_dim == 80) return launch_d<80>(tm, p, plan, grid, bf16, stream);
  return RB_E_UNSUPPORTED;
}

}  // namespace rb
