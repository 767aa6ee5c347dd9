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

}  // namespace b2f

using namespace b2f;

extern "C" {

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
