// Fused MoE combine + residual add + RMSNorm of one token row per CTA (shared
// by the decode-step kernels and the expert-parallel peer exchange).
#pragma once
#include "common.cuh"

namespace b2f {

template <int NW>
__device__ __forceinline__ float block_sum(float v, float* sh) {
  v = warp_sum<32>(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = 0.f;
  const int nw = int(blockDim.x + 31) >> 5;
  for (int w = 0; w < nw && w < NW; ++w) t += sh[w];
  __syncthreads();
  return t;
}

// h = resid + sum_j score[m, j] * y[m*k + j]  (y may be null -> h = resid;
// scores may be null -> every score is 1)
// resid_out = bf16(h); norm_out = bf16(w * h_bf16 * rsqrt(mean(h_bf16^2) + eps))
// One CTA per row; a thread owns chunks of 8 contiguous elements (16-byte loads).
constexpr int CMB_CHUNKS = 4;

constexpr int CMB_BATCH = 8;  // expert rows / partial planes whose loads are issued together

__device__ __forceinline__ void combine_rmsnorm_block(
    const __nv_bfloat16* __restrict__ resid, const __nv_bfloat16* __restrict__ y,
    const float* __restrict__ scores, int k, const __nv_bfloat16* __restrict__ w, float eps, int H,
    __nv_bfloat16* __restrict__ resid_out, __nv_bfloat16* __restrict__ norm_out,
    const float* __restrict__ partial, int nsplit, int64_t M) {
  __shared__ float sh[8];
  const int64_t m = blockIdx.x;
  const int nvec = H / 8;
  float hv[CMB_CHUNKS][8];
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < CMB_CHUNKS; ++q) {
    const int v = threadIdx.x + q * blockDim.x;
    if (v >= nvec) break;
    const uint4 rr = reinterpret_cast<const uint4*>(resid + m * H)[v];
    const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr);
    float h[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h[2 * i] = __low2float(r2[i]);
      h[2 * i + 1] = __high2float(r2[i]);
    }
    if (partial) {  // split-K fp32 partials of a projection added to the residual
      // all planes' loads in flight before the first add (in plane order)
      for (int j0 = 0; j0 < nsplit; j0 += CMB_BATCH) {
        float4 a[CMB_BATCH], c[CMB_BATCH];
#pragma unroll
        for (int u = 0; u < CMB_BATCH; ++u) {
          if (j0 + u < nsplit) {
            const float4* pp = reinterpret_cast<const float4*>(partial + (int64_t(j0 + u) * M + m) * H) + 2 * v;
            a[u] = pp[0];
            c[u] = pp[1];
          }
        }
#pragma unroll
        for (int u = 0; u < CMB_BATCH; ++u) {
          if (j0 + u < nsplit) {
            h[0] += a[u].x;
            h[1] += a[u].y;
            h[2] += a[u].z;
            h[3] += a[u].w;
            h[4] += c[u].x;
            h[5] += c[u].y;
            h[6] += c[u].z;
            h[7] += c[u].w;
          }
        }
      }
    }
    if (y) {
      for (int j0 = 0; j0 < k; j0 += CMB_BATCH) {
        uint4 yy[CMB_BATCH];
        float sc[CMB_BATCH];
#pragma unroll
        for (int u = 0; u < CMB_BATCH; ++u) {
          if (j0 + u < k) {
            sc[u] = scores ? scores[m * k + j0 + u] : 1.0f;
            yy[u] = reinterpret_cast<const uint4*>(y + (m * k + j0 + u) * H)[v];
          }
        }
#pragma unroll
        for (int u = 0; u < CMB_BATCH; ++u) {
          if (j0 + u < k) {
            const __nv_bfloat162* y2 = reinterpret_cast<const __nv_bfloat162*>(&yy[u]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              h[2 * i] += sc[u] * __low2float(y2[i]);
              h[2 * i + 1] += sc[u] * __high2float(y2[i]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      hv[q][i] = __bfloat162float(__float2bfloat16_rn(h[i]));
      ss += hv[q][i] * hv[q][i];
    }
  }
  const float tot = block_sum<8>(ss, sh);
  const float rs = rsqrtf(tot / float(H) + eps);
#pragma unroll
  for (int q = 0; q < CMB_CHUNKS; ++q) {
    const int v = threadIdx.x + q * blockDim.x;
    if (v >= nvec) break;
    const uint4 ww = reinterpret_cast<const uint4*>(w)[v];
    const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&ww);
    uint32_t o[4], ro[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[i] = pack_bf16x2(__low2float(w2[i]) * hv[q][2 * i] * rs, __high2float(w2[i]) * hv[q][2 * i + 1] * rs);
      ro[i] = pack_bf16x2(hv[q][2 * i], hv[q][2 * i + 1]);
    }
    if (resid_out) reinterpret_cast<uint4*>(resid_out + m * H)[v] = make_uint4(ro[0], ro[1], ro[2], ro[3]);
    reinterpret_cast<uint4*>(norm_out + m * H)[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace b2f
