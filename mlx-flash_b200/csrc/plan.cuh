// MoE plan: counting sort of routed assignments by expert, cut into tiles.
//
// Shared by the single-GPU plan (b2f_moe_plan: expert ids straight from the
// router's top-k) and the expert-parallel plan (b2f_ep_plan: expert ids read
// from every rank's gathered routing segment, experts owned by other ranks
// skipped).  One CTA of 1024 threads: A is at most a few tens of thousands
// of assignments per step, so the sort is a few microseconds.
//
// Workspace layout (PlanLayout):
//   hdr     int32[16]   hdr[0] = number of slots, hdr[1] = status,
//                       hdr[2] = arrival counter of the fused top-k + plan kernel
//   counts  int32[E]    assignments per expert
//   offsets int32[E+1]  exclusive scan of counts
//   cursor  int32[E]    scatter cursors
//   soff    int32[E+1]  slots of the experts before each expert (exclusive scan)
//   sorted  int32[A]    assignment ids grouped by expert
//   slots   int4[S]     {expert, begin in sorted, count <= tile, 0}: the slots
//                       holding more than tile/2 assignments first, then the
//                       rest, each part in expert order (E <= 1024; else all
//                       in expert order) -- grids launched over the slots then
//                       start their longest CTAs first, so the last wave holds
//                       short ones
#pragma once
#include "common.cuh"

namespace b2f {

struct PlanLayout {
  int64_t off_hdr, off_counts, off_offsets, off_cursor, off_soff, off_sorted, off_slots, total;
};

static inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

static inline int64_t plan_max_slots(int64_t A, int64_t E, int tile) {
  const int64_t ne = A < E ? A : E;
  return ne + A / tile + 1;
}

static inline PlanLayout plan_layout(int64_t A, int64_t E, int tile) {
  PlanLayout L;
  int64_t o = 0;
  L.off_hdr = o;
  o += 64;
  L.off_counts = o;
  o = align_up(o + 4 * E, 16);
  L.off_offsets = o;
  o = align_up(o + 4 * (E + 1), 16);
  L.off_cursor = o;
  o = align_up(o + 4 * E, 16);
  L.off_soff = o;
  o = align_up(o + 4 * (E + 1), 16);
  L.off_sorted = o;
  o = align_up(o + 4 * (A > 0 ? A : 1), 16);
  L.off_slots = o;
  o = align_up(o + 16 * plan_max_slots(A, E, tile), 256);
  L.total = o;
  return L;
}

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024).
static __device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int t = lane < nw ? warp_tot[lane] : 0;
    int ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, ti, o);
      if (lane >= o) ti += n;
    }
    if (lane < nw) warp_tot[lane] = ti - t;
    if (lane == nw - 1) *total = ti;
  }
  __syncthreads();
  const int r = inc - v + warp_tot[warp];
  __syncthreads();
  return r;
}

// Expert ids given directly: any id outside [0, E) is an error.
struct DenseExperts {
  const int32_t* expert_of;
  __device__ __forceinline__ int expert(int a) const { return expert_of[a]; }
  __device__ __forceinline__ bool invalid(int a, int e, int E) const { return e < 0 || e >= E; }
  __device__ __forceinline__ void side(int a, int e, int E) const {}
};

// Expert ids read from W gathered routing segments (expert parallelism).
// Segment r (seg_bytes long) holds rank r's T tokens: bf16 rows of the
// normalised hidden state at byte 0 (row pitch row_bytes), then int32
// top-k ids [T, k] at inds_off and float32 scores [T, k] at scores_off.
// Assignment a = (r*T + t)*k + j.  Experts [e_begin, e_begin + E) are this
// rank's; others are skipped.  Side outputs per assignment: the gathered x
// row, the score (0 for foreign experts) and the local expert (-1 foreign).
struct GatheredExperts {
  const char* recv;
  int64_t seg_bytes, inds_off, scores_off, seg_rows;
  int T, k, e_begin, e_total;
  int32_t* x_row;
  float* wts;
  int32_t* local;
  __device__ __forceinline__ int global_expert(int a) const {
    const int tk = T * k;
    const int r = a / tk, rem = a - r * tk;
    return reinterpret_cast<const int32_t*>(recv + r * seg_bytes + inds_off)[rem];
  }
  __device__ __forceinline__ int expert(int a) const { return global_expert(a) - e_begin; }
  __device__ __forceinline__ bool invalid(int a, int e, int E) const {
    const int g = e + e_begin;
    return g < 0 || g >= e_total;
  }
  __device__ __forceinline__ void side(int a, int e, int E) const {
    const int tk = T * k;
    const int r = a / tk, rem = a - r * tk, t = rem / k;
    const bool mine = e >= 0 && e < E;
    x_row[a] = int32_t(r * seg_rows + t);
    wts[a] = mine ? reinterpret_cast<const float*>(recv + r * seg_bytes + scores_off)[rem] : 0.0f;
    local[a] = mine ? e : -1;
  }
};

// Expert ids carried in the rows an all-to-all dispatch delivered: received
// row r (pitch `pitch` bytes) holds the token's bf16 hidden row (H values),
// then int32 local expert ids [k] (-1 where that slot's expert lives on
// another rank) at meta_off, then float32 scores [k] at meta_off + 4k.
// Assignment a = r*k + j.  Side outputs as for GatheredExperts.
struct A2AExperts {
  const char* recv;
  int64_t pitch, meta_off;
  int k;
  int32_t* x_row;
  float* wts;
  int32_t* local;
  __device__ __forceinline__ int expert(int a) const {
    const int r = a / k, j = a - r * k;
    return reinterpret_cast<const int32_t*>(recv + int64_t(r) * pitch + meta_off)[j];
  }
  __device__ __forceinline__ bool invalid(int a, int e, int E) const { return e < -1 || e >= E; }
  __device__ __forceinline__ void side(int a, int e, int E) const {
    const int r = a / k, j = a - r * k;
    const bool mine = e >= 0 && e < E;
    x_row[a] = r;
    wts[a] = mine ? reinterpret_cast<const float*>(recv + int64_t(r) * pitch + meta_off + 4 * k)[j] : 0.0f;
    local[a] = mine ? e : -1;
  }
};

// The counting sort, run by one whole thread block (any blockDim <= 1024).
// Per-expert counters live in shared memory (E <= PLAN_SMEM_E) so the
// count / scan / scatter phases cost shared-memory atomics and block
// barriers only; larger E falls back to the workspace arrays.
constexpr int PLAN_SMEM_E = 1024;

template <class Src>
__device__ __forceinline__ void moe_plan_block(const Src& src, int A, int E, int tile, char* ws, PlanLayout L,
                                               int32_t* status_out) {
  int32_t* hdr = reinterpret_cast<int32_t*>(ws + L.off_hdr);
  int32_t* g_counts = reinterpret_cast<int32_t*>(ws + L.off_counts);
  int32_t* g_offsets = reinterpret_cast<int32_t*>(ws + L.off_offsets);
  int32_t* g_cursor = reinterpret_cast<int32_t*>(ws + L.off_cursor);
  int32_t* g_soff = reinterpret_cast<int32_t*>(ws + L.off_soff);
  int32_t* sorted = reinterpret_cast<int32_t*>(ws + L.off_sorted);
  int4* slots = reinterpret_cast<int4*>(ws + L.off_slots);
  __shared__ int warp_tot[32];
  __shared__ int total;
  __shared__ int bad;
  __shared__ int s_counts[PLAN_SMEM_E], s_cursor[PLAN_SMEM_E], s_offsets[PLAN_SMEM_E + 1], s_soff[PLAN_SMEM_E + 1];
  __shared__ int s_hoff[PLAN_SMEM_E];  // first heavy slot of each expert
  __shared__ int heavy_total;
  const bool sm = E <= PLAN_SMEM_E;
  int32_t* counts = sm ? s_counts : g_counts;
  int32_t* cursor = sm ? s_cursor : g_cursor;
  int32_t* offsets = sm ? s_offsets : g_offsets;
  int32_t* soff = sm ? s_soff : g_soff;
  if (threadIdx.x == 0) bad = 0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    counts[e] = 0;
    cursor[e] = 0;
  }
  __syncthreads();
  for (int a = threadIdx.x; a < A; a += blockDim.x) {
    const int e = src.expert(a);
    if (src.invalid(a, e, E)) bad = 1;
    src.side(a, e, E);
    if (e >= 0 && e < E) atomicAdd(&counts[e], 1);
  }
  __syncthreads();
  // exclusive scans over experts (chunks of blockDim.x): assignments, slots,
  // heavy slots (more than tile/2 assignments: every full slot and a last
  // slot past half a tile)
  int run = 0, srun = 0, hrun = 0;
  for (int base = 0; base < E; base += blockDim.x) {
    const int e = base + threadIdx.x;
    const int cnt = e < E ? counts[e] : 0;
    const int ns = (cnt + tile - 1) / tile;
    const int nfull = cnt / tile;
    const int nh = nfull + (cnt - nfull * tile > tile / 2 ? 1 : 0);
    const int ex = block_exclusive_scan(cnt, warp_tot, &total);
    const int t1 = total;
    __syncthreads();
    const int sx = block_exclusive_scan(ns, warp_tot, &total);
    const int t2 = total;
    __syncthreads();
    const int hx = block_exclusive_scan(nh, warp_tot, &total);
    const int t3 = total;
    if (e < E) {
      offsets[e] = run + ex;
      soff[e] = srun + sx;
      if (sm) s_hoff[e] = hrun + hx;
    }
    run += t1;
    srun += t2;
    hrun += t3;
    __syncthreads();
  }
  if (threadIdx.x == 0) heavy_total = hrun;
  if (threadIdx.x == 0) {
    offsets[E] = run;
    soff[E] = srun;
    hdr[0] = srun;
    hdr[1] = bad ? B2F_ERR_INVALID : B2F_OK;
    if (status_out) *status_out = hdr[1];
  }
  __syncthreads();
  for (int a = threadIdx.x; a < A; a += blockDim.x) {
    const int e = src.expert(a);
    if (e >= 0 && e < E) {
      const int pos = offsets[e] + atomicAdd(&cursor[e], 1);
      sorted[pos] = a;
    }
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int cnt = counts[e];
    for (int j = 0; j * tile < cnt; ++j) {
      const int c = min(tile, cnt - j * tile);
      // heavy slots of expert e are its first ones (j < its heavy count); its
      // light slot (at most one, the last) follows all heavy slots, after
      // the light slots of the experts before it (soff[e] - s_hoff[e])
      int s = soff[e] + j;
      if (sm) s = c > tile / 2 ? s_hoff[e] + j : heavy_total + soff[e] - s_hoff[e];
      slots[s] = make_int4(e, offsets[e] + j * tile, c, 0);
    }
  }
  if (sm) {  // the per-expert arrays of the workspace layout, for readers of the plan
    for (int e = threadIdx.x; e <= E; e += blockDim.x) {
      if (e < E) {
        g_counts[e] = counts[e];
        g_cursor[e] = cursor[e];
      }
      g_offsets[e] = offsets[e];
      g_soff[e] = soff[e];
    }
  }
}

template <class Src>
__global__ void __launch_bounds__(1024) moe_plan_kernel(const Src src, int A, int E, int tile, char* ws,
                                                        PlanLayout L, int32_t* status_out) {
  pdl_enter();
  moe_plan_block(src, A, E, tile, ws, L, status_out);
}

}  // namespace b2f
