// (e) Expert parallelism: the device-side halves of dispatch and combine.
//
// Expert parallelism over W ranks (one process per GPU).  Rank r owns the
// contiguous expert block [e_begin, e_begin + e_count) of the ExpertShard
// partition (distributed_experts.py:36-80: floor(E/W) experts per rank, the
// last rank takes the remainder).  Attention and the router run per rank on
// the rank's own T tokens; a decode step's MoE block then is
//
//   dispatch  every rank's routing segment {x rows, top-k ids, scores} is
//             gathered onto every rank (one NCCL all-gather of W segments);
//   plan      b2f_ep_plan: counting sort of the W*T*k gathered assignments by
//             LOCAL expert, skipping experts owned elsewhere, plus per
//             assignment the gathered x row, its score and its local expert;
//   experts   b2f_gather_qgemm_affine_tcgen05 / b2f_gather_qgemv_affine on
//             the local expert shard, x read in place from the gathered
//             segments through the x-row index;
//   partial   b2f_ep_combine_partial: per gathered token the score-weighted
//             sum of its local expert outputs (0 where it has none);
//   combine   one NCCL reduce-scatter (sum) hands every rank the sum over
//             ranks of its own tokens' partials = the full MoE output.
//
// With T tokens per rank the all-gather moves W*T rows per rank, the same
// bytes as a fixed-capacity all-to-all with capacity T per peer (a token is
// sent to a peer once, whatever number of its k experts that peer owns); it
// needs no host-side count exchange, so the whole step stays inside one
// CUDA graph.
#include "common.cuh"
#include "plan.cuh"

namespace b2f {

// out[g, :] = sum_j (local[g*k+j] >= 0) * wts[g*k+j] * y[g*k+j, :]
// One CTA per gathered token; a thread owns chunks of 8 contiguous columns.
__global__ void __launch_bounds__(256) ep_combine_partial_kernel(
    const __nv_bfloat16* __restrict__ y, int64_t ldy, const float* __restrict__ wts,
    const int32_t* __restrict__ local, int k, int H, __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int64_t g = blockIdx.x;
  __shared__ float w_s[64];
  __shared__ int n_s;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int j = 0; j < k; ++j) {
      const int64_t a = g * k + j;
      if (local[a] >= 0) {
        w_s[n] = wts[a];
        w_s[32 + n] = __int_as_float(j);
        ++n;
      }
    }
    n_s = n;
  }
  __syncthreads();
  const int n = n_s;
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int i = 0; i < n; ++i) {
      const float sc = w_s[i];
      const int j = __float_as_int(w_s[32 + i]);
      const uint4 yy = reinterpret_cast<const uint4*>(y + (g * k + j) * ldy)[v];
      const __nv_bfloat162* y2 = reinterpret_cast<const __nv_bfloat162*>(&yy);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += sc * __low2float(y2[q]);
        acc[2 * q + 1] += sc * __high2float(y2[q]);
      }
    }
    uint4 o;
    uint32_t* o32 = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) o32[q] = pack_bf16x2(acc[2 * q], acc[2 * q + 1]);
    reinterpret_cast<uint4*>(out + g * ldo)[v] = o;
  }
}

// ---------------------------------------------------------------------------
// All-to-all expert parallelism (prefill-sized batches): every token goes once
// to each rank that owns at least one of its k experts, as one row
//   [bf16 hidden row H][int32 local expert ids k][float32 scores k] (pitch bytes)
// in a send buffer grouped by destination rank (token order inside a group),
// so one all_to_all_single with per-rank byte splits carries ids, scores and
// activations together.  Ownership is the ExpertShard block partition:
// floor(E/W) experts per rank, the last rank takes the remainder.

__device__ __forceinline__ int shard_owner(int e, int per, int W) { return min(e / per, W - 1); }

// One CTA (1024 threads): per destination d, the tokens with an expert on d
// get consecutive send positions (token order): pos[t*W + d] = base_d + rank
// of t among them, or -1; counts[d] = tokens sent to d.
__global__ void __launch_bounds__(1024) ep_a2a_positions_kernel(const int32_t* __restrict__ inds, int T, int k, int W,
                                                                 int e_total, int32_t* __restrict__ pos,
                                                                 int32_t* __restrict__ counts,
                                                                 int32_t* __restrict__ status) {
  __shared__ int warp_tot[32];
  __shared__ int total;
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  const int per = e_total / W;
  int base = 0;
  for (int d = 0; d < W; ++d) {
    int run = 0;
    for (int t0 = 0; t0 < T; t0 += blockDim.x) {
      const int t = t0 + threadIdx.x;
      int f = 0;
      if (t < T) {
        for (int j = 0; j < k; ++j) {
          const int e = inds[int64_t(t) * k + j];
          if (e < 0 || e >= e_total) {
            bad = 1;
            continue;
          }
          f |= shard_owner(e, per, W) == d;
        }
      }
      const int ex = block_exclusive_scan(f, warp_tot, &total);
      const int tot = total;
      if (t < T) pos[int64_t(t) * W + d] = f ? base + run + ex : -1;
      run += tot;
      __syncthreads();
    }
    if (threadIdx.x == 0) counts[d] = run;
    base += run;
  }
  __syncthreads();
  if (threadIdx.x == 0 && status) *status = bad ? B2F_ERR_INVALID : B2F_OK;
}

// One CTA per (token, destination) with a send position: the hidden row and
// the token's local ids / scores for that destination.
__global__ void __launch_bounds__(256) ep_a2a_pack_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                          const int32_t* __restrict__ inds,
                                                          const float* __restrict__ scores, const int32_t* pos, int T,
                                                          int k, int W, int e_total, int H, char* __restrict__ send,
                                                          int64_t pitch) {
  const int64_t td = blockIdx.x;
  const int t = int(td / W), d = int(td - int64_t(t) * W);
  const int p = pos[td];
  if (p < 0) return;
  char* row = send + int64_t(p) * pitch;
  const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(t) * ldx);
  uint4* dst = reinterpret_cast<uint4*>(row);
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) dst[v] = src[v];
  if (threadIdx.x < k) {
    const int per = e_total / W;
    const int j = threadIdx.x;
    const int e = inds[int64_t(t) * k + j];
    const bool mine = e >= 0 && e < e_total && shard_owner(e, per, W) == d;
    reinterpret_cast<int32_t*>(row + 2 * int64_t(H))[j] = mine ? e - d * per : -1;
    reinterpret_cast<float*>(row + 2 * int64_t(H) + 4 * k)[j] = mine ? scores[int64_t(t) * k + j] : 0.f;
  }
}

// out[t] = (resid[t]) + sum over d (ascending) of ret[pos[t*W + d]] -- the
// partial sums the owner ranks returned for token t, f32 accumulation.
__global__ void __launch_bounds__(256) ep_a2a_combine_kernel(const __nv_bfloat16* __restrict__ ret, int64_t ldr,
                                                             const int32_t* __restrict__ pos, int W, int H,
                                                             const __nv_bfloat16* __restrict__ resid,
                                                             __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int64_t t = blockIdx.x;
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    if (resid) {
      const uint4 rr = reinterpret_cast<const uint4*>(resid + t * ldo)[v];
      const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] = __low2float(r2[q]);
        acc[2 * q + 1] = __high2float(r2[q]);
      }
    }
    for (int d = 0; d < W; ++d) {
      const int p = pos[t * W + d];
      if (p < 0) continue;
      const uint4 yy = reinterpret_cast<const uint4*>(ret + int64_t(p) * ldr)[v];
      const __nv_bfloat162* y2 = reinterpret_cast<const __nv_bfloat162*>(&yy);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += __low2float(y2[q]);
        acc[2 * q + 1] += __high2float(y2[q]);
      }
    }
    uint4 o;
    uint32_t* o32 = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) o32[q] = pack_bf16x2(acc[2 * q], acc[2 * q + 1]);
    reinterpret_cast<uint4*>(out + t * ldo)[v] = o;
  }
}

}  // namespace b2f

using namespace b2f;

extern "C" {

int64_t b2f_ep_a2a_row_pitch(int64_t H, int64_t k) {
  if (H <= 0 || k <= 0) return 0;
  return align_up(2 * H + 8 * k, 16);
}

int b2f_ep_a2a_dispatch(const void* x, int64_t ldx, const int32_t* inds, const float* scores, int64_t T, int64_t k,
                        int64_t W, int64_t e_total, int64_t H, void* send, int64_t send_bytes, int32_t* pos,
                        int32_t* send_counts, int32_t* status_out, void* stream) {
  if (T < 0 || k <= 0 || k > 32 || W <= 0 || W > 64 || H <= 0 || H % 8 != 0) return B2F_ERR_INVALID;
  if (T > 0 && (ldx < H || ldx % 8 != 0)) return B2F_ERR_INVALID;  // a rank without tokens reads no row
  if (e_total < W) return B2F_ERR_INVALID;  // every rank owns at least one expert
  if (T * W > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  if (!pos || !send_counts) return B2F_ERR_INVALID;
  const int64_t pitch = b2f_ep_a2a_row_pitch(H, k);
  const int64_t cap = T * (W < k ? W : k);  // a token goes to at most min(W, k) ranks
  if (T > 0 && (!x || !inds || !scores || !send)) return B2F_ERR_INVALID;
  if (send_bytes < cap * pitch) return B2F_ERR_WORKSPACE;
  if (!aligned(x, 16) || !aligned(send, 16)) return B2F_ERR_ALIGN;
  cudaStream_t st = as_stream(stream);
  ep_a2a_positions_kernel<<<1, 1024, 0, st>>>(inds, int(T), int(k), int(W), int(e_total), pos, send_counts,
                                              status_out);
  int rc = check_launch();
  if (rc != B2F_OK || T == 0) return rc;
  ep_a2a_pack_kernel<<<unsigned(T * W), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), ldx, inds, scores, pos,
                                                      int(T), int(k), int(W), int(e_total), int(H),
                                                      static_cast<char*>(send), pitch);
  return check_launch();
}

int b2f_ep_a2a_plan(const void* recv, int64_t R, int64_t H, int64_t k, int64_t e_count, int tile, int32_t* x_row,
                    float* wts, int32_t* local, void* workspace, int64_t workspace_bytes, int32_t* status_out,
                    void* stream) {
  if (R < 0 || H <= 0 || H % 8 != 0 || k <= 0 || k > 32 || e_count <= 0) return B2F_ERR_INVALID;
  if (tile < 8 || tile > 256 || tile % 8 != 0) return B2F_ERR_INVALID;
  const int64_t A = R * k;
  if (A > 0x3fffffff || e_count > 65535) return B2F_ERR_UNSUPPORTED;
  PlanLayout L = plan_layout(A, e_count, tile);
  if (!workspace || workspace_bytes < L.total) return B2F_ERR_WORKSPACE;
  if (A > 0 && (!recv || !x_row || !wts || !local)) return B2F_ERR_INVALID;
  if (!aligned(workspace, 16) || (A > 0 && !aligned(recv, 16))) return B2F_ERR_ALIGN;
  A2AExperts src;
  src.recv = static_cast<const char*>(recv);
  src.pitch = b2f_ep_a2a_row_pitch(H, k);
  src.meta_off = 2 * H;
  src.k = int(k);
  src.x_row = x_row;
  src.wts = wts;
  src.local = local;
  moe_plan_kernel<<<1, 1024, 0, as_stream(stream)>>>(src, int(A), int(e_count), tile,
                                                     static_cast<char*>(workspace), L, status_out);
  return check_launch();
}

int b2f_ep_a2a_combine(const void* ret, int64_t ldr, const int32_t* pos, int64_t T, int64_t W, int64_t H,
                       const void* resid, void* out, int64_t ldo, void* stream) {
  if (T < 0 || W <= 0 || W > 64 || H <= 0 || H % 8 != 0 || ldr < H || ldo < H) return B2F_ERR_INVALID;
  if (ldr % 8 || ldo % 8) return B2F_ERR_ALIGN;
  if (T == 0) return B2F_OK;
  if (!pos || !out) return B2F_ERR_INVALID;
  if ((ret && !aligned(ret, 16)) || !aligned(out, 16) || (resid && !aligned(resid, 16))) return B2F_ERR_ALIGN;
  if (T > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  const int threads = int(H / 8 < 256 ? ((H / 8 + 31) / 32) * 32 : 256);
  ep_a2a_combine_kernel<<<unsigned(T), threads, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(ret), ldr, pos, int(W), int(H), static_cast<const __nv_bfloat16*>(resid),
      static_cast<__nv_bfloat16*>(out), ldo);
  return check_launch();
}

int b2f_ep_plan(const void* recv, int64_t seg_bytes, int64_t row_bytes, int64_t inds_off, int64_t scores_off,
                int64_t W, int64_t T, int64_t k, int64_t e_begin, int64_t e_count, int64_t e_total, int tile,
                int32_t* x_row, float* wts, int32_t* local, void* workspace, int64_t workspace_bytes,
                int32_t* status_out, void* stream) {
  if (W <= 0 || T < 0 || k <= 0 || k > 32 || e_count <= 0 || e_begin < 0 || e_begin + e_count > e_total)
    return B2F_ERR_INVALID;
  if (tile < 8 || tile > 256 || tile % 8 != 0) return B2F_ERR_INVALID;
  if (row_bytes <= 0 || seg_bytes <= 0 || seg_bytes % row_bytes != 0) return B2F_ERR_INVALID;
  if (inds_off < 0 || scores_off < 0 || inds_off % 4 || scores_off % 4) return B2F_ERR_ALIGN;
  if (inds_off + 4 * T * k > seg_bytes || scores_off + 4 * T * k > seg_bytes || T * row_bytes > inds_off)
    return B2F_ERR_INVALID;
  const int64_t A = W * T * k;
  if (A > 0x3fffffff || e_count > 65535 || W * (seg_bytes / row_bytes) > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  PlanLayout L = plan_layout(A, e_count, tile);
  if (!workspace || workspace_bytes < L.total) return B2F_ERR_WORKSPACE;
  if (A > 0 && (!recv || !x_row || !wts || !local)) return B2F_ERR_INVALID;
  if (!aligned(workspace, 16) || !aligned(recv, 16)) return B2F_ERR_ALIGN;
  GatheredExperts src;
  src.recv = static_cast<const char*>(recv);
  src.seg_bytes = seg_bytes;
  src.inds_off = inds_off;
  src.scores_off = scores_off;
  src.seg_rows = seg_bytes / row_bytes;
  src.T = int(T);
  src.k = int(k);
  src.e_begin = int(e_begin);
  src.e_total = int(e_total);
  src.x_row = x_row;
  src.wts = wts;
  src.local = local;
  moe_plan_kernel<<<1, 1024, 0, as_stream(stream)>>>(src, int(A), int(e_count), tile,
                                                     static_cast<char*>(workspace), L, status_out);
  return check_launch();
}

int b2f_ep_combine_partial(const void* y, int64_t ldy, const float* wts, const int32_t* local, int64_t G,
                           int64_t k, int64_t H, void* out, int64_t ldo, void* stream) {
  if (G < 0 || k <= 0 || k > 32 || H <= 0 || H % 8 != 0 || ldy < H || ldo < H) return B2F_ERR_INVALID;
  if (ldy % 8 || ldo % 8) return B2F_ERR_ALIGN;
  if (G == 0) return B2F_OK;
  if (!y || !wts || !local || !out) return B2F_ERR_INVALID;
  if (!aligned(y, 16) || !aligned(out, 16)) return B2F_ERR_ALIGN;
  if (G > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  const int threads = int(H / 8 < 256 ? ((H / 8 + 31) / 32) * 32 : 256);
  ep_combine_partial_kernel<<<unsigned(G), threads, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(y), ldy, wts, local, int(k), int(H), static_cast<__nv_bfloat16*>(out),
      ldo);
  return check_launch();
}

}  // extern "C"
