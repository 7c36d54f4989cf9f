// moe.cu — mixture-of-experts routing, token dispatch and combine.
//
// The device form of the reference's MoE layer around the expert GEMMs
// (`route`, src/clef/model.rs:462-489; `Buckets::build` / `combine`,
// src/clef/engine.rs:284-340):
//
//   route     softmax over the E router logits of a token, top-k by
//             probability (ties to the lower expert id), weights renormalised
//             over the selected k (in selection order, f32);
//   dispatch  per-expert row counts, 256-row-aligned expert segments in a
//             permuted activation buffer (one CTA-pair tile of the grouped
//             GEMM never spans two experts), the 128-row tile -> expert
//             table the grouped GEMM reads, and the gather of each routed
//             token row;
//   combine   x[t] += w_j * y[row_j] over the token's k experts in ascending
//             expert id (f32, product then sum, as the reference).
//
// Rows inside an expert's segment are placed by atomics, so their order
// varies between calls; every row's result is independent of its position
// and the combine reads rows through the slot -> row map, so outputs do not.
//
// Workspace (int32 words, laid out by moe_layout):
//   counts[E]  seg_start[E+1]  cursor[E]  tile_expert[max_tiles]
//   row_of_slot[T*k]  token_of_row[max_rows]
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "sm100.cuh"

namespace rb {

constexpr int kMoeSeg = 256;   // expert segment alignment = grouped-GEMM CTA-pair M tile
constexpr int kMoeTile = 128;  // rows per tile_expert entry = one CTA's M rows

MoeLayout moe_layout(int64_t tokens, int top_k, int experts) {
  MoeLayout L{};
  L.max_rows = ((tokens * top_k + static_cast<int64_t>(experts) * (kMoeSeg - 1)) + kMoeSeg - 1) / kMoeSeg *
               kMoeSeg;
  L.max_tiles = L.max_rows / kMoeTile;
  int64_t off = 0;
  L.counts = off; off += experts;
  L.seg_start = off; off += experts + 1;
  L.cursor = off; off += experts;
  L.tile_expert = off; off += L.max_tiles;
  L.row_of_slot = off; off += tokens * top_k;
  L.token_of_row = off; off += L.max_rows;
  L.words = off;
  return L;
}

// ---------------------------------------------------------------- route
// One warp per token; lane l holds logits l, l+32, ... (EPL per lane).
template <int EPL>
__global__ void moe_route_kernel(const float* __restrict__ logits, int64_t tokens, int E, int k, int norm,
                                 int32_t* __restrict__ ids, float* __restrict__ wts) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); t < tokens; t += nw) {
    float p[EPL];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      p[i] = e < E ? logits[t * E + e] : -INFINITY;
      m = fmaxf(m, p[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      p[i] = (lane + 32 * i) < E ? expf(p[i] - m) : 0.0f;
      s += p[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
    for (int i = 0; i < EPL; ++i) p[i] = (lane + 32 * i) < E ? __fdiv_rn(p[i], s) : -1.0f;
    // k rounds of a warp arg-max; ties go to the lower expert id.
    float sel[32];
    int sel_id[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      if (r >= k) break;
      float bv = -2.0f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const int e = lane + 32 * i;
        if (p[i] > bv || (p[i] == bv && e < bi)) { bv = p[i]; bi = e; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      sel[r] = bv;
      sel_id[r] = bi;
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (lane + 32 * i == bi) p[i] = -1.0f;
    }
    if (lane == 0) {
      float sum = 0.0f;
#pragma unroll
      for (int r = 0; r < 32; ++r)
        if (r < k) sum = __fadd_rn(sum, sel[r]);
#pragma unroll
      for (int r = 0; r < 32; ++r) {
        if (r < k) {
          ids[t * k + r] = sel_id[r];
          wts[t * k + r] = norm ? __fdiv_rn(sel[r], sum) : sel[r];
        }
      }
    }
  }
}

int launch_moe_route(const float* logits, int64_t tokens, int experts, int top_k, int norm, int32_t* ids,
                     float* wts, cudaStream_t st) {
  if (experts < 1 || experts > 256 || top_k < 1 || top_k > 32 || top_k > experts) return RB_E_SHAPE;
  int64_t g = (tokens + 7) / 8;
  if (g > 148 * 16) g = 148 * 16;
  if (g < 1) g = 1;
  const int blocks = static_cast<int>(g);
  if (experts <= 32) moe_route_kernel<1><<<blocks, 256, 0, st>>>(logits, tokens, experts, top_k, norm, ids, wts);
  else if (experts <= 64) moe_route_kernel<2><<<blocks, 256, 0, st>>>(logits, tokens, experts, top_k, norm, ids, wts);
  else if (experts <= 128) moe_route_kernel<4><<<blocks, 256, 0, st>>>(logits, tokens, experts, top_k, norm, ids, wts);
  else moe_route_kernel<8><<<blocks, 256, 0, st>>>(logits, tokens, experts, top_k, norm, ids, wts);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

// ---------------------------------------------------------------- dispatch
// Count and scatter split the slots into one contiguous chunk per block and
// aggregate in shared memory first: one global atomic per (block, expert)
// instead of one per slot (the slots of a popular expert would otherwise
// serialise on its counter).
__device__ __forceinline__ void slot_chunk(int64_t slots, int64_t& s0, int64_t& s1) {
  const int64_t chunk = (slots + gridDim.x - 1) / gridDim.x;
  s0 = blockIdx.x * chunk;
  s1 = s0 + chunk < slots ? s0 + chunk : slots;
}

__global__ void moe_count_kernel(const int32_t* __restrict__ ids, int64_t slots, int E, int32_t* counts,
                                 uint32_t* err) {
  __shared__ int32_t s_cnt[1024];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  int64_t s0, s1;
  slot_chunk(slots, s0, s1);
  for (int64_t s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
    const int e = ids[s];
    if (e == -1) continue;  // no expert: a padding row of a fixed-capacity exchange
    if (e < 0 || e >= E) {
      atomicOr(err, kErrBadShape);
      continue;
    }
    atomicAdd(&s_cnt[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    if (s_cnt[e]) atomicAdd(&counts[e], s_cnt[e]);
}

// One block: exclusive scan of the 256-aligned segment sizes, the segment
// starts, the insertion cursors and the 128-row tile -> expert table.
__global__ void moe_offsets_kernel(const int32_t* __restrict__ counts, int E, int64_t max_tiles,
                                   int32_t* seg_start, int32_t* cursor, int32_t* tile_expert) {
  __shared__ int32_t s_start[1025];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_start[e] = (counts[e] + kMoeSeg - 1) / kMoeSeg * kMoeSeg;
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t acc = 0;
    for (int e = 0; e < E; ++e) {
      const int32_t sz = s_start[e];
      s_start[e] = acc;
      acc += sz;
    }
    s_start[E] = acc;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) {
    seg_start[e] = s_start[e];
    if (e < E) cursor[e] = s_start[e];
  }
  const int64_t used = s_start[E] / kMoeTile;
  for (int64_t mt = threadIdx.x; mt < max_tiles; mt += blockDim.x) {
    int32_t ex = -1;
    if (mt < used) {
      // expert whose segment holds tile mt (binary search over the starts)
      int lo = 0, hi = E - 1;
      const int32_t row = static_cast<int32_t>(mt * kMoeTile);
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_start[mid] <= row) lo = mid; else hi = mid - 1;
      }
      // skip empty segments that start at the same row
      while (lo + 1 < E && s_start[lo + 1] <= row) ++lo;
      ex = lo;
    }
    tile_expert[mt] = ex;
  }
}

// Pass 1 ranks each slot among its block's slots of the same expert (kept in
// row_of_slot), one global atomic per expert then reserves the block's rows,
// pass 2 turns ranks into rows. Each thread revisits only its own slots.
__global__ void moe_scatter_kernel(const int32_t* __restrict__ ids, int64_t slots, int k, int E, int32_t* cursor,
                                   int32_t* row_of_slot, int32_t* token_of_row) {
  __shared__ int32_t s_cnt[1024];
  __shared__ int32_t s_base[1024];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  int64_t s0, s1;
  slot_chunk(slots, s0, s1);
  for (int64_t s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
    const int e = ids[s];
    if (e < 0 || e >= E) continue;
    row_of_slot[s] = atomicAdd(&s_cnt[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    if (s_cnt[e]) s_base[e] = atomicAdd(&cursor[e], s_cnt[e]);
  __syncthreads();
  for (int64_t s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
    const int e = ids[s];
    if (e < 0 || e >= E) {
      row_of_slot[s] = -1;  // no row (a padding slot): gathers and combines skip it
      continue;
    }
    const int32_t row = s_base[e] + row_of_slot[s];
    row_of_slot[s] = row;
    token_of_row[row] = static_cast<int32_t>(s / k);
  }
}

// One warp per permuted row: copy the routed token's f16 row, or zeros for
// the padding rows of a segment. Rows of unused tiles are left alone (the
// grouped GEMM skips those tiles). The padding rows' outputs are never read,
// but the grouped GEMMs measured 1.5-3% faster on zero padding rows than on
// stale data (they run under the power cap), which more than repays the
// zero writes.
__global__ void moe_gather_kernel(const __half* __restrict__ x, int64_t hidden, int64_t max_rows,
                                  const int32_t* __restrict__ counts, const int32_t* __restrict__ seg_start,
                                  const int32_t* __restrict__ tile_expert, const int32_t* __restrict__ token_of_row,
                                  __half* __restrict__ xp) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t v8 = hidden / 8;
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); r < max_rows; r += nw) {
    const int e = tile_expert[r / kMoeTile];
    if (e < 0) continue;
    uint4* dst = reinterpret_cast<uint4*>(xp + r * hidden);
    if (r - seg_start[e] >= counts[e]) {  // segment padding
#pragma unroll 8
      for (int64_t i = lane; i < v8; i += 32) __stcs(dst + i, make_uint4(0u, 0u, 0u, 0u));
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(token_of_row[r]) * hidden);
#pragma unroll 8
    for (int64_t i = lane; i < v8; i += 32) __stcs(dst + i, __ldg(src + i));  // loads in flight together
  }
}

int launch_moe_dispatch(const int32_t* ids, int64_t tokens, int top_k, int experts, const void* x, int64_t hidden,
                        int32_t* ws, void* x_perm, uint32_t* err, cudaStream_t st) {
  if (experts < 1 || experts > 1024 || hidden % 8) return RB_E_SHAPE;
  const MoeLayout L = moe_layout(tokens, top_k, experts);
  const int64_t slots = tokens * top_k;
  if (cudaMemsetAsync(ws + L.counts, 0, sizeof(int32_t) * experts, st) != cudaSuccess) return RB_E_DEVICE;
  int64_t g = (slots + 2047) / 2048;  // ~8 slots a thread
  if (g > 148) g = 148;
  if (g < 1) g = 1;
  moe_count_kernel<<<static_cast<int>(g), 256, 0, st>>>(ids, slots, experts, ws + L.counts, err);
  moe_offsets_kernel<<<1, 256, 0, st>>>(ws + L.counts, experts, L.max_tiles, ws + L.seg_start, ws + L.cursor,
                                        ws + L.tile_expert);
  moe_scatter_kernel<<<static_cast<int>(g), 256, 0, st>>>(ids, slots, top_k, experts, ws + L.cursor,
                                                          ws + L.row_of_slot, ws + L.token_of_row);
  int64_t gr = (L.max_rows + 7) / 8;
  if (gr > 148 * 16) gr = 148 * 16;
  moe_gather_kernel<<<static_cast<int>(gr), 256, 0, st>>>(
      reinterpret_cast<const __half*>(x), hidden, L.max_rows, ws + L.counts, ws + L.seg_start, ws + L.tile_expert,
      ws + L.token_of_row, reinterpret_cast<__half*>(x_perm));
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

// ---------------------------------------------------------------- combine
// One warp per token: x[t] (f32, in place) += w_j * y[row_j] over the
// token's k slots in ascending expert id; each lane owns 8-column groups.
template <int KMAX>
__global__ void moe_combine_kernel(float* __restrict__ x, const __half* __restrict__ y, int64_t hidden,
                                   const int32_t* __restrict__ ids, const float* __restrict__ wts,
                                   const int32_t* __restrict__ row_of_slot, int64_t tokens, int k) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); t < tokens; t += nw) {
    // slot j of this token lives in lane j; rank = position in ascending expert order
    int my_e = 0x7fffffff, my_row = 0;
    float my_w = 0.0f;
    if (lane < k) {
      my_e = ids[t * k + lane];
      my_w = wts[t * k + lane];
      my_row = row_of_slot[t * k + lane];
    }
    int rank = 0;
    for (int j = 0; j < k; ++j) {
      const int ej = __shfl_sync(0xffffffffu, my_e, j);
      if (ej < my_e || (ej == my_e && j < lane)) ++rank;
    }
    // order[r] = lane holding rank r
    int ord_row[KMAX];
    float ord_w[KMAX];
#pragma unroll
    for (int r = 0; r < KMAX; ++r) {
      if (r >= k) break;
      const unsigned hit = __ballot_sync(0xffffffffu, lane < k && rank == r);
      const int src = __ffs(hit) - 1;
      ord_row[r] = __shfl_sync(0xffffffffu, my_row, src);
      ord_w[r] = __shfl_sync(0xffffffffu, my_w, src);
    }
    float* xr = x + t * hidden;
#pragma unroll 2
    for (int64_t c = lane * 8; c < hidden; c += 256) {
      float4 a0 = *reinterpret_cast<const float4*>(xr + c);
      float4 a1 = *reinterpret_cast<const float4*>(xr + c + 4);
      float acc[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      uint4 uv[KMAX];
#pragma unroll
      for (int r = 0; r < KMAX; ++r)  // all of the token's rows in flight
        if (r < k && ord_row[r] >= 0)
          uv[r] = __ldg(reinterpret_cast<const uint4*>(y + static_cast<int64_t>(ord_row[r]) * hidden + c));
#pragma unroll
      for (int r = 0; r < KMAX; ++r) {
        if (r >= k) break;
        if (ord_row[r] < 0) continue;  // a slot that overflowed its exchange buffer (flagged)
        const uint4 u = uv[r];
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __half22float2(h[q]);
          acc[2 * q] = __fadd_rn(acc[2 * q], __fmul_rn(f.x, ord_w[r]));
          acc[2 * q + 1] = __fadd_rn(acc[2 * q + 1], __fmul_rn(f.y, ord_w[r]));
        }
      }
      *reinterpret_cast<float4*>(xr + c) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(xr + c + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

int launch_moe_combine(float* x, const void* y, int64_t hidden, const int32_t* ids, const float* wts,
                       const int32_t* ws, int64_t tokens, int top_k, int experts, cudaStream_t st) {
  if (hidden % 8 || top_k > 32) return RB_E_SHAPE;
  const MoeLayout L = moe_layout(tokens, top_k, experts);
  int64_t g = (tokens + 7) / 8;
  if (g > 148 * 16) g = 148 * 16;
  if (g < 1) g = 1;
  if (top_k <= 8)
    moe_combine_kernel<8><<<static_cast<int>(g), 256, 0, st>>>(x, reinterpret_cast<const __half*>(y), hidden, ids,
                                                              wts, ws + L.row_of_slot, tokens, top_k);
  else
    moe_combine_kernel<32><<<static_cast<int>(g), 256, 0, st>>>(x, reinterpret_cast<const __half*>(y), hidden, ids,
                                                               wts, ws + L.row_of_slot, tokens, top_k);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

// ---------------------------------------------------------------- expert parallelism
// Send-side bookkeeping for an all-to-all token exchange: the destination of
// slot (t, j) is the rank owning expert ids[t, j] (experts_per_rank
// consecutive ids per rank). Slots are grouped by destination in the send
// buffer; for each: the token's f16 row, the expert id local to the
// destination, and (kept here) the send position of every slot for the
// combine after the outputs come back.
__global__ void ep_count_kernel(const int32_t* __restrict__ ids, int64_t slots, int per_rank, int ranks,
                                int32_t* dest_counts, uint32_t* err) {
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < slots;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int q = ids[s] / per_rank;
    if (ids[s] < 0 || q >= ranks) {
      atomicOr(err, kErrBadShape);
      continue;
    }
    atomicAdd(&dest_counts[q], 1);
  }
}

__global__ void ep_offsets_kernel(const int32_t* __restrict__ dest_counts, int ranks, int32_t* dest_cursor) {
  if (threadIdx.x == 0) {
    int32_t acc = 0;
    for (int q = 0; q < ranks; ++q) {
      dest_cursor[q] = acc;
      acc += dest_counts[q];
    }
  }
}

__global__ void ep_scatter_kernel(const int32_t* __restrict__ ids, int64_t slots, int k, int per_rank,
                                  int32_t* dest_cursor, int32_t* send_meta, int32_t* slot_pos) {
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < slots;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = ids[s];
    const int q = e / per_rank;
    const int32_t pos = atomicAdd(&dest_cursor[q], 1);
    send_meta[pos] = e - q * per_rank;
    slot_pos[s] = pos;
  }
}

// rows_out[i] = rows_in[idx[i] / div] (f16 rows, one warp per output row).
__global__ void gather_rows_kernel(const __half* __restrict__ in, const int32_t* __restrict__ idx, int div,
                                   int64_t n, int64_t hidden, __half* __restrict__ out, int inverse) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t v8 = hidden / 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += nw) {
    // forward: out[idx[i]] = in[i / div] (scatter by slot position);
    // inverse: out[i] = in[idx[i]] (gather).
    const int64_t src = inverse ? idx[i] : i / div;
    const int64_t dst = inverse ? i : idx[i];
    if (src < 0 || dst < 0) continue;  // a padding or overflowed slot: nothing to move
    const uint4* a = reinterpret_cast<const uint4*>(in + src * hidden);
    uint4* b = reinterpret_cast<uint4*>(out + dst * hidden);
#pragma unroll 8
    for (int64_t c = lane; c < v8; c += 32) b[c] = __ldg(a + c);  // loads in flight together
  }
}

int launch_ep_build_send(const int32_t* ids, int64_t tokens, int top_k, int experts, int ranks, const void* x,
                         int64_t hidden, int32_t* dest_counts, int32_t* dest_cursor, int32_t* send_meta,
                         int32_t* slot_pos, void* send_rows, uint32_t* err, cudaStream_t st) {
  if (ranks < 1 || experts % ranks || hidden % 8) return RB_E_SHAPE;
  const int per_rank = experts / ranks;
  const int64_t slots = tokens * top_k;
  if (cudaMemsetAsync(dest_counts, 0, sizeof(int32_t) * ranks, st) != cudaSuccess) return RB_E_DEVICE;
  int64_t g = (slots + 255) / 256;
  if (g > 148 * 8) g = 148 * 8;
  if (g < 1) g = 1;
  ep_count_kernel<<<static_cast<int>(g), 256, 0, st>>>(ids, slots, per_rank, ranks, dest_counts, err);
  ep_offsets_kernel<<<1, 32, 0, st>>>(dest_counts, ranks, dest_cursor);
  ep_scatter_kernel<<<static_cast<int>(g), 256, 0, st>>>(ids, slots, top_k, per_rank, dest_cursor, send_meta,
                                                         slot_pos);
  int64_t gr = (slots + 7) / 8;
  if (gr > 148 * 16) gr = 148 * 16;
  gather_rows_kernel<<<static_cast<int>(gr), 256, 0, st>>>(reinterpret_cast<const __half*>(x), slot_pos, top_k,
                                                           slots, hidden, reinterpret_cast<__half*>(send_rows), 0);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

// Fixed-capacity form: destination q owns send positions [q*cap, (q+1)*cap),
// so every all-to-all split is `cap` rows and no count has to reach the host.
// A slot beyond its destination's capacity is not sent (slot_pos = -1) and
// flags kErrOverflow; unused positions keep send_meta = -1 (no expert).
__global__ void ep_offsets_fixed_kernel(const int32_t* __restrict__ dest_counts, int ranks, int cap,
                                        int32_t* dest_cursor, uint32_t* err) {
  for (int q = threadIdx.x; q < ranks; q += blockDim.x) {
    dest_cursor[q] = q * cap;
    if (dest_counts[q] > cap) atomicOr(err, kErrOverflow);
  }
}

__global__ void ep_scatter_fixed_kernel(const int32_t* __restrict__ ids, int64_t slots, int per_rank, int cap,
                                        int32_t* dest_cursor, int32_t* send_meta, int32_t* slot_pos) {
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < slots;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = ids[s];
    const int q = e / per_rank;
    const int32_t pos = atomicAdd(&dest_cursor[q], 1);
    if (pos >= (q + 1) * cap) {
      slot_pos[s] = -1;
      continue;
    }
    send_meta[pos] = e - q * per_rank;
    slot_pos[s] = pos;
  }
}

int launch_ep_build_send_fixed(const int32_t* ids, int64_t tokens, int top_k, int experts, int ranks, int cap,
                               const void* x, int64_t hidden, int32_t* dest_counts, int32_t* dest_cursor,
                               int32_t* send_meta, int32_t* slot_pos, void* send_rows, uint32_t* err,
                               cudaStream_t st) {
  if (ranks < 1 || experts % ranks || hidden % 8 || cap < 1) return RB_E_SHAPE;
  const int per_rank = experts / ranks;
  const int64_t slots = tokens * top_k;
  if (cudaMemsetAsync(dest_counts, 0, sizeof(int32_t) * ranks, st) != cudaSuccess ||
      cudaMemsetAsync(send_meta, 0xFF, sizeof(int32_t) * static_cast<size_t>(ranks) * cap, st) != cudaSuccess)
    return RB_E_DEVICE;
  int64_t g = (slots + 255) / 256;
  if (g > 148 * 8) g = 148 * 8;
  if (g < 1) g = 1;
  ep_count_kernel<<<static_cast<int>(g), 256, 0, st>>>(ids, slots, per_rank, ranks, dest_counts, err);
  ep_offsets_fixed_kernel<<<1, 256, 0, st>>>(dest_counts, ranks, cap, dest_cursor, err);
  ep_scatter_fixed_kernel<<<static_cast<int>(g), 256, 0, st>>>(ids, slots, per_rank, cap, dest_cursor, send_meta,
                                                               slot_pos);
  int64_t gr = (slots + 7) / 8;
  if (gr > 148 * 16) gr = 148 * 16;
  gather_rows_kernel<<<static_cast<int>(gr), 256, 0, st>>>(reinterpret_cast<const __half*>(x), slot_pos, top_k,
                                                           slots, hidden, reinterpret_cast<__half*>(send_rows), 0);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

int launch_gather_rows(const void* in, const int32_t* idx, int64_t n, int64_t hidden, void* out, cudaStream_t st) {
  if (hidden % 8) return RB_E_SHAPE;
  int64_t g = (n + 7) / 8;
  if (g > 148 * 16) g = 148 * 16;
  if (g < 1) g = 1;
  gather_rows_kernel<<<static_cast<int>(g), 256, 0, st>>>(reinterpret_cast<const __half*>(in), idx, 1, n, hidden,
                                                          reinterpret_cast<__half*>(out), 1);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

int launch_moe_combine_rows(float* x, const void* y, int64_t hidden, const int32_t* ids, const float* wts,
                            const int32_t* row_of_slot, int64_t tokens, int top_k, cudaStream_t st) {
  if (hidden % 8 || top_k > 32) return RB_E_SHAPE;
  int64_t g = (tokens + 7) / 8;
  if (g > 148 * 16) g = 148 * 16;
  if (g < 1) g = 1;
  if (top_k <= 8)
    moe_combine_kernel<8><<<static_cast<int>(g), 256, 0, st>>>(x, reinterpret_cast<const __half*>(y), hidden, ids,
                                                              wts, row_of_slot, tokens, top_k);
  else
    moe_combine_kernel<32><<<static_cast<int>(g), 256, 0, st>>>(x, reinterpret_cast<const __half*>(y), hidden, ids,
                                                               wts, row_of_slot, tokens, top_k);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

}  // namespace rb
