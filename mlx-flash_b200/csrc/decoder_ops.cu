// Small fused kernels around the quantized hot path of a Qwen3-MoE-shaped
// decode step: RMSNorm (optionally fused with the MoE combine and the
// residual add), per-head QK-RMSNorm + RoPE + quantized KV append into the
// paged cache, softmax top-k routing, and a row argmax.  All are
// bandwidth/latency-bound; one CTA per token row.
#include "common.cuh"

namespace b2f {

template <int NW>
__device__ __forceinline__ float block_sum(float v, float* sh) {
  v = warp_sum<32>(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) t += sh[w];
  __syncthreads();
  return t;
}

// h = resid + sum_j score[m, j] * y[m*k + j]  (y may be null -> h = resid)
// resid_out = bf16(h); norm_out = bf16(w * h_bf16 * rsqrt(mean(h_bf16^2) + eps))
__global__ void __launch_bounds__(256) combine_rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ resid, const __nv_bfloat16* __restrict__ y,
    const float* __restrict__ scores, int k, const __nv_bfloat16* __restrict__ w, float eps, int H,
    __nv_bfloat16* __restrict__ resid_out, __nv_bfloat16* __restrict__ norm_out) {
  __shared__ float sh[8];
  const int64_t m = blockIdx.x;
  float hv[16];
  float ss = 0.f;
  int n = 0;
  for (int i = threadIdx.x; i < H; i += blockDim.x, ++n) {
    float h = __bfloat162float(resid[m * H + i]);
    if (y) {
      for (int j = 0; j < k; ++j) h += scores[m * k + j] * __bfloat162float(y[(m * k + j) * H + i]);
    }
    const float hb = __bfloat162float(__float2bfloat16_rn(h));
    if (n < 16) hv[n] = hb;
    ss += hb * hb;
  }
  const float tot = block_sum<8>(ss, sh);
  const float r = rsqrtf(tot / float(H) + eps);
  n = 0;
  for (int i = threadIdx.x; i < H; i += blockDim.x, ++n) {
    const float hb = hv[n];
    if (resid_out) resid_out[m * H + i] = __float2bfloat16_rn(hb);
    norm_out[m * H + i] = __float2bfloat16_rn(__bfloat162float(w[i]) * hb * r);
  }
}

// Per token: q heads get RMSNorm(q_norm) + RoPE -> q_out; k heads RMSNorm(k_norm)
// + RoPE -> bf16 -> reference KV quantizer -> page slot; v heads quantized as is.
// qkv row layout: [Hq*D | Hkv*D | Hkv*D].  Rotary: NeoX half rotation,
// inv_freq_i = theta^(-2i/D).  D = 128; one warp per head (4 values per lane,
// d = lane + 32*i, so d and d+64 sit in the same lane).
struct RopeKvParams {
  const __nv_bfloat16* qkv;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  float eps, theta;
  const int32_t* positions;
  __nv_bfloat16* q_out;
  uint8_t* k_codes;
  float* k_scales;
  uint8_t* v_codes;
  float* v_scales;
  const int32_t* block_table;
  int64_t max_pages;
  int Hq, Hkv, PS, bits;
};

__global__ void __launch_bounds__(256) qk_norm_rope_kv_kernel(const RopeKvParams p) {
  constexpr int D = 128;
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int NH = p.Hq + 2 * p.Hkv;
  const int pos = p.positions[b];
  const int page = p.block_table[int64_t(b) * p.max_pages + pos / p.PS];
  const int slot = pos % p.PS;
  const __nv_bfloat16* row = p.qkv + int64_t(b) * NH * D;
  const float mi = p.bits == 8 ? 127.f : 7.f;
  for (int h = warp; h < NH; h += nw) {
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(row[h * D + lane + 32 * i]);
    const bool is_q = h < p.Hq, is_k = !is_q && h < p.Hq + p.Hkv;
    if (is_q || is_k) {
      const __nv_bfloat16* nw_ = is_q ? p.q_norm : p.k_norm;
      float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
      ss = warp_sum<32>(ss);
      const float r = rsqrtf(ss / float(D) + p.eps);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        v[i] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(nw_[lane + 32 * i]) * v[i] * r));
      // rotary: pairs (d, d+64) -> (i=0,i=2), (i=1,i=3)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int d = lane + 32 * i;  // frequency index < 64
        const float inv = exp2f(-(2.f * float(d) / float(D)) * log2f(p.theta));
        float sn, cs;
        sincosf(float(pos) * inv, &sn, &cs);
        const float x1 = v[i], x2 = v[i + 2];
        v[i] = __bfloat162float(__float2bfloat16_rn(x1 * cs - x2 * sn));
        v[i + 2] = __bfloat162float(__float2bfloat16_rn(x2 * cs + x1 * sn));
      }
    }
    if (is_q) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        p.q_out[(int64_t(b) * p.Hq + h) * D + lane + 32 * i] = __float2bfloat16_rn(v[i]);
      continue;
    }
    // quantize (bf16 semantics, groups of 64: i in {0,1} -> group 0, {2,3} -> group 1)
    const int kvh = is_k ? h - p.Hq : h - p.Hq - p.Hkv;
    uint8_t* codes = is_k ? p.k_codes : p.v_codes;
    float* scales = is_k ? p.k_scales : p.v_scales;
    const int64_t rrow = int64_t(page) * p.Hkv * p.PS + int64_t(kvh) * p.PS + slot;
    const int RB = D * p.bits / 8;
    uint32_t c[4];
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      float m = fmaxf(fabsf(v[2 * g]), fabsf(v[2 * g + 1]));
      m = warp_max<32>(m);
      float scale = TagBF16::round(__fdiv_rn(m, mi));
      if (scale == 0.f) scale = 1.f;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float xs = TagBF16::round(__fdiv_rn(v[2 * g + e], scale));
        float xq = TagBF16::round(rintf(xs));
        xq = fminf(fmaxf(xq, -mi), mi);
        c[2 * g + e] = uint32_t(int(TagBF16::round(xq + mi)));
      }
      if (lane == 0) scales[rrow * 2 + g] = scale;
    }
    uint8_t* dst = codes + rrow * RB;
    if (p.bits == 8) {
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = uint8_t(c[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t nxt = __shfl_down_sync(0xffffffffu, c[i], 1);
        if ((lane & 1) == 0) dst[(lane + 32 * i) >> 1] = uint8_t((c[i] << 4) | (nxt & 0xF));
      }
    }
  }
}

// logits[t, e] = x[t].wr[e] (+ bias[e]); gates = softmax; top-k by value
// (ties -> lower id); scores optionally renormalised over the top-k.
// CTA = 4 tokens x 8 warps; x rows staged in shared memory.
constexpr int ROUTE_TOK = 4;

__global__ void __launch_bounds__(256) route_topk_kernel(const __nv_bfloat16* __restrict__ x, int T, int H,
                                                         const __nv_bfloat16* __restrict__ wr,
                                                         const float* __restrict__ bias, int E, int k,
                                                         int renorm, int32_t* __restrict__ inds,
                                                         float* __restrict__ scores) {
  extern __shared__ float sm[];
  float* xs = sm;                      // [ROUTE_TOK][H]
  float* lg = sm + ROUTE_TOK * H;      // [ROUTE_TOK][E]
  const int t0 = blockIdx.x * ROUTE_TOK;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int i = threadIdx.x; i < ROUTE_TOK * H; i += blockDim.x) {
    const int t = i / H, d = i % H;
    xs[i] = (t0 + t < T) ? __bfloat162float(x[int64_t(t0 + t) * H + d]) : 0.f;
  }
  __syncthreads();
  for (int e = warp; e < E; e += nw) {
    float acc[ROUTE_TOK] = {0.f, 0.f, 0.f, 0.f};
    const __nv_bfloat16* wrow = wr + int64_t(e) * H;
    for (int d = lane * 2; d < H; d += 64) {
      const __nv_bfloat162 w2 = *reinterpret_cast<const __nv_bfloat162*>(wrow + d);
      const float w0 = __low2float(w2), w1 = __high2float(w2);
#pragma unroll
      for (int t = 0; t < ROUTE_TOK; ++t) acc[t] += w0 * xs[t * H + d] + w1 * xs[t * H + d + 1];
    }
#pragma unroll
    for (int t = 0; t < ROUTE_TOK; ++t) {
      const float s = warp_sum<32>(acc[t]);
      if (lane == 0) lg[t * E + e] = s + (bias ? bias[e] : 0.f);
    }
  }
  __syncthreads();
  if (warp < ROUTE_TOK && t0 + warp < T) {
    const int t = warp;
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, lg[t * E + e]);
    mx = warp_max<32>(mx);
    float sum = 0.f;
    for (int e = lane; e < E; e += 32) {
      const float g = expf(lg[t * E + e] - mx);
      lg[t * E + e] = g;
      sum += g;
    }
    sum = warp_sum<32>(sum);
    float picked = 0.f;
    int64_t base = int64_t(t0 + t) * k;
    for (int j = 0; j < k; ++j) {
      float bv = -1.f;
      int bi = 0x7fffffff;
      for (int e = lane; e < E; e += 32) {
        const float g = lg[t * E + e];
        if (g > bv || (g == bv && e < bi)) {
          bv = g;
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        inds[base + j] = bi;
        scores[base + j] = bv / sum;
        lg[t * E + bi] = -2.f;  // remove from the candidates
      }
      picked += bv / sum;
      __syncwarp();
    }
    if (renorm && lane < k) scores[base + lane] = scores[base + lane] / picked;
  }
}

__global__ void __launch_bounds__(256) argmax_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t V,
                                                          int32_t* __restrict__ out) {
  __shared__ float sv[8];
  __shared__ int si[8];
  const int64_t m = blockIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = __bfloat162float(x[m * V + i]);
    if (v > bv) {
      bv = v;
      bi = int(i);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < int(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
        bv = sv[w];
        bi = si[w];
      }
    out[m] = bi;
  }
}

}  // namespace b2f

using namespace b2f;

extern "C" {

int b2f_combine_rmsnorm(const void* resid, const void* y, const float* scores, int64_t M, int64_t k,
                        const void* weight, float eps, int64_t H, void* resid_out, void* norm_out,
                        void* stream) {
  if (M < 0 || H <= 0 || H > 16 * 256 || (y && (k <= 0 || !scores))) return B2F_ERR_INVALID;
  if (M == 0) return B2F_OK;
  if (!resid || !weight || !norm_out) return B2F_ERR_INVALID;
  combine_rmsnorm_kernel<<<unsigned(M), 256, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(resid), static_cast<const __nv_bfloat16*>(y), scores, int(k),
      static_cast<const __nv_bfloat16*>(weight), eps, int(H), static_cast<__nv_bfloat16*>(resid_out),
      static_cast<__nv_bfloat16*>(norm_out));
  return check_launch();
}

int b2f_qk_norm_rope_kv_append(const void* qkv, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                               const void* q_norm, const void* k_norm, float eps, float rope_theta,
                               const int32_t* positions, void* q_out, uint8_t* k_codes, float* k_scales,
                               uint8_t* v_codes, float* v_scales, const int32_t* block_table,
                               int64_t max_pages, int64_t page_size, int bits, void* stream) {
  if (D != 128) return B2F_ERR_UNSUPPORTED;
  if (!(bits == 4 || bits == 8)) return B2F_ERR_UNSUPPORTED;
  if (B < 0 || Hq <= 0 || Hkv <= 0 || page_size <= 0 || max_pages <= 0) return B2F_ERR_INVALID;
  if (B == 0) return B2F_OK;
  if (!qkv || !q_norm || !k_norm || !positions || !q_out || !k_codes || !k_scales || !v_codes ||
      !v_scales || !block_table)
    return B2F_ERR_INVALID;
  RopeKvParams p{};
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.q_norm = static_cast<const __nv_bfloat16*>(q_norm);
  p.k_norm = static_cast<const __nv_bfloat16*>(k_norm);
  p.eps = eps;
  p.theta = rope_theta;
  p.positions = positions;
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.k_codes = k_codes;
  p.k_scales = k_scales;
  p.v_codes = v_codes;
  p.v_scales = v_scales;
  p.block_table = block_table;
  p.max_pages = max_pages;
  p.Hq = int(Hq);
  p.Hkv = int(Hkv);
  p.PS = int(page_size);
  p.bits = bits;
  qk_norm_rope_kv_kernel<<<unsigned(B), 256, 0, as_stream(stream)>>>(p);
  return check_launch();
}

int b2f_moe_route_topk(const void* x, int64_t T, int64_t H, const void* wr, const float* bias, int64_t E,
                       int64_t k, int renorm, int32_t* inds, float* scores, void* stream) {
  if (T < 0 || H <= 0 || H % 2 || E <= 0 || k <= 0 || k > E || k > 32) return B2F_ERR_INVALID;
  if (T == 0) return B2F_OK;
  if (!x || !wr || !inds || !scores) return B2F_ERR_INVALID;
  const int64_t smem = (ROUTE_TOK * H + ROUTE_TOK * E) * int64_t(sizeof(float));
  if (smem > 200 * 1024) return B2F_ERR_UNSUPPORTED;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(route_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return B2F_ERR_CUDA;
    }
  }
  const unsigned grid = unsigned((T + ROUTE_TOK - 1) / ROUTE_TOK);
  route_topk_kernel<<<grid, 256, smem, as_stream(stream)>>>(static_cast<const __nv_bfloat16*>(x), int(T), int(H),
                                                            static_cast<const __nv_bfloat16*>(wr), bias, int(E),
                                                            int(k), renorm, inds, scores);
  return check_launch();
}

int b2f_argmax_rows(const void* x, int64_t M, int64_t V, int32_t* out, void* stream) {
  if (M < 0 || V <= 0 || V > 0x7fffffff) return B2F_ERR_INVALID;
  if (M == 0) return B2F_OK;
  if (!x || !out) return B2F_ERR_INVALID;
  argmax_rows_kernel<<<unsigned(M), 256, 0, as_stream(stream)>>>(static_cast<const __nv_bfloat16*>(x), V, out);
  return check_launch();
}

}  // extern "C"
