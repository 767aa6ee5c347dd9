// Small fused kernels around the quantized hot path of a Qwen3-MoE-shaped
// decode step: RMSNorm (optionally fused with the MoE combine and the
// residual add), per-head QK-RMSNorm + RoPE + quantized KV append into the
// paged cache, softmax top-k routing, and a row argmax.  All are
// bandwidth/latency-bound; one CTA per token row.
#include "common.cuh"
#include "norm.cuh"
#include "plan.cuh"

namespace b2f {

__global__ void __launch_bounds__(256) combine_rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ resid, const __nv_bfloat16* __restrict__ y,
    const float* __restrict__ scores, int k, const __nv_bfloat16* __restrict__ w, float eps, int H,
    __nv_bfloat16* __restrict__ resid_out, __nv_bfloat16* __restrict__ norm_out,
    const float* __restrict__ partial = nullptr, int nsplit = 0, int64_t M = 0) {
  pdl_enter();
  combine_rmsnorm_block(resid, y, scores, k, w, eps, H, resid_out, norm_out, partial, nsplit, M);
}

// Per token: q heads get RMSNorm(q_norm) + RoPE -> q_out; k heads RMSNorm(k_norm)
// + RoPE -> bf16 -> reference KV quantizer -> page slot; v heads quantized as is.
// qkv row layout: [Hq*D | Hkv*D | Hkv*D].  Rotary: NeoX half rotation,
// inv_freq_i = theta^(-2i/D).  D = 128; one warp per head (4 values per lane,
// d = lane + 32*i, so d and d+64 sit in the same lane).
struct RopeKvParams {
  const __nv_bfloat16* qkv;
  const float* qkv_partial;  // split-K fp32 partials [nsplit][B][NH*D] (replaces qkv when set)
  int nsplit;
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

// grid (B, heads / 8): one warp per head of the token, so the (Hq + 2Hkv)
// heads of a decode batch spread over many SMs instead of queuing on B CTAs.
__global__ void __launch_bounds__(256) qk_norm_rope_kv_kernel(const RopeKvParams p) {
  pdl_enter();
  constexpr int D = 128;
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int NH = p.Hq + 2 * p.Hkv;
  const int pos = p.positions[b];
  const int page = p.block_table[int64_t(b) * p.max_pages + pos / p.PS];
  const int slot = pos % p.PS;
  const __nv_bfloat16* row = p.qkv + int64_t(b) * NH * D;
  const float mi = p.bits == 8 ? 127.f : p.bits == 4 ? 7.f : 1.f;
  // rotary angles of this token: one sincosf per frequency, shared by all heads
  __shared__ float rope_c[D / 2], rope_s[D / 2];
  if (threadIdx.x < D / 2) {
    const float inv = exp2f(-(2.f * float(threadIdx.x) / float(D)) * log2f(p.theta));
    sincosf(float(pos) * inv, &rope_s[threadIdx.x], &rope_c[threadIdx.x]);
  }
  __syncthreads();
  for (int h = blockIdx.y * nw + warp; h < min(NH, int(blockIdx.y + 1) * nw); h += nw) {
    float v[4];
    if (p.qkv_partial) {
      // the projection's bf16 output, formed here from its split-K partials
      const int64_t plane = int64_t(gridDim.x) * NH * D;
      float a[4] = {0.f, 0.f, 0.f, 0.f};
      const float* base = p.qkv_partial + int64_t(b) * NH * D + h * D + lane;
      for (int j0 = 0; j0 < p.nsplit; j0 += 8) {
        float t[8][4];  // eight planes' loads in flight, summed in plane order
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
          for (int i = 0; i < 4; ++i) t[u][i] = j0 + u < p.nsplit ? base[(j0 + u) * plane + 32 * i] : 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (j0 + u < p.nsplit) a[i] += t[u][i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(__float2bfloat16_rn(a[i]));
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(row[h * D + lane + 32 * i]);
    }
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
        const float sn = rope_s[d], cs = rope_c[d];
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
    } else if (p.bits == 2) {
      // four codes per byte, the first in the top two bits
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t c1 = __shfl_down_sync(0xffffffffu, c[i], 1);
        const uint32_t c2 = __shfl_down_sync(0xffffffffu, c[i], 2);
        const uint32_t c3 = __shfl_down_sync(0xffffffffu, c[i], 3);
        if ((lane & 3) == 0)
          dst[(lane + 32 * i) >> 2] = uint8_t((c[i] << 6) | ((c1 & 3u) << 4) | ((c2 & 3u) << 2) | (c3 & 3u));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t nxt = __shfl_down_sync(0xffffffffu, c[i], 1);
        if ((lane & 1) == 0) dst[(lane + 32 * i) >> 1] = uint8_t((c[i] << 4) | (nxt & 0xF));
      }
    }
  }
}

// logits[t, e] = x[t].wr[e] (+ bias[e]): CTA = 8 experts x 8 tokens, one warp
// per expert.  The CTA's 8 token rows are staged in shared memory with
// coalesced 16-byte loads; each warp first issues all of its router-row
// loads (RL_MAXV 16-byte vectors per lane, H <= 8192), then reads x from
// shared memory, so one memory latency covers the whole dot product.
constexpr int RL_TOK = 8;
constexpr int RL_MAXV = 4;  // router-row vectors per lane per pass (1024 elements per warp pass)

__global__ void __launch_bounds__(256) route_logits_kernel(const __nv_bfloat16* __restrict__ x, int T, int H,
                                                           const __nv_bfloat16* __restrict__ wr,
                                                           const float* __restrict__ bias, int E,
                                                           float* __restrict__ logits, int32_t* __restrict__ counter) {
  pdl_enter();
  // the MoE plan's arrival counter, read by the routing kernel that follows
  if (counter && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *counter = 0;
  extern __shared__ __align__(16) uint4 xs[];  // [RL_TOK][H/8]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e = blockIdx.x * 8 + warp;
  const int t0 = blockIdx.y * RL_TOK;
  const int nt = min(RL_TOK, T - t0);
  const int hv = H / 8;
  for (int i = threadIdx.x; i < RL_TOK * hv; i += blockDim.x) {
    const int t = i / hv, v = i - t * hv;
    xs[i] = t < nt ? reinterpret_cast<const uint4*>(x + int64_t(t0 + t) * H)[v] : make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
  if (e >= E) return;
  float acc[RL_TOK];
#pragma unroll
  for (int t = 0; t < RL_TOK; ++t) acc[t] = 0.f;
  const uint4* wrow = reinterpret_cast<const uint4*>(wr + int64_t(e) * H);
  for (int v0 = 0; v0 < hv; v0 += 32 * RL_MAXV) {
    uint4 wv[RL_MAXV];
#pragma unroll
    for (int j = 0; j < RL_MAXV; ++j) {
      const int v = v0 + lane + 32 * j;
      wv[j] = v < hv ? wrow[v] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < RL_MAXV; ++j) {
      const int v = v0 + lane + 32 * j;
      if (v >= hv) break;
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wv[j]);
      float wf[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        wf[2 * i] = __low2float(w2[i]);
        wf[2 * i + 1] = __high2float(w2[i]);
      }
#pragma unroll
      for (int t = 0; t < RL_TOK; ++t) {
        const uint4 xv = xs[t * hv + v];
        const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          acc[t] = fmaf(wf[2 * i], __low2float(x2[i]), fmaf(wf[2 * i + 1], __high2float(x2[i]), acc[t]));
      }
    }
  }
#pragma unroll
  for (int t = 0; t < RL_TOK; ++t) {
    const float v = warp_sum<32>(acc[t]);
    if (lane == 0 && t < nt) logits[int64_t(t0 + t) * E + e] = v + (bias ? bias[e] : 0.f);
  }
}

// The same logits on warp-level tensor-core MMA (bf16 products, fp32 sums):
// CTA = 16 tokens x 8 experts, its 8 warps each take 1/8 of H in 32-wide
// chunks (lane (r, c) holds k in [8c, 8c+8) of a chunk, the nibble-free
// version of the pair order the expert GEMM uses), and the 8 partial tiles
// are summed in a fixed order through shared memory.  E % 8 == 0,
// H % 256 == 0.
__global__ void __launch_bounds__(256) route_logits_mma_kernel(const __nv_bfloat16* __restrict__ x, int T, int H,
                                                               const __nv_bfloat16* __restrict__ wr,
                                                               const float* __restrict__ bias, int E,
                                                               float* __restrict__ logits, int32_t* __restrict__ counter) {
  pdl_enter();
  // the MoE plan's arrival counter, read by the routing kernel that follows
  if (counter && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *counter = 0;
  __shared__ float red[8][32][4];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = lane >> 2, c = lane & 3;
  const int e0 = blockIdx.x * 8, t0 = blockIdx.y * 16;
  const int kw = H / 8;  // K range of this warp
  const int k0 = warp * kw;
  const bool v0 = t0 + r < T, v1 = t0 + r + 8 < T;
  const __nv_bfloat16* xr0 = x + int64_t(v0 ? t0 + r : 0) * H + k0 + 8 * c;
  const __nv_bfloat16* xr1 = x + int64_t(v1 ? t0 + r + 8 : 0) * H + k0 + 8 * c;
  const __nv_bfloat16* wrow = wr + int64_t(e0 + r) * H + k0 + 8 * c;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  constexpr int U = 4;  // chunks in flight
  for (int ch = 0; ch < kw / 32; ch += U) {
    uint4 a0[U], a1[U], bw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const bool in = ch + u < kw / 32;
      const int o = 32 * (ch + u);
      a0[u] = (in && v0) ? *reinterpret_cast<const uint4*>(xr0 + o) : make_uint4(0u, 0u, 0u, 0u);
      a1[u] = (in && v1) ? *reinterpret_cast<const uint4*>(xr1 + o) : make_uint4(0u, 0u, 0u, 0u);
      bw[u] = in ? *reinterpret_cast<const uint4*>(wrow + o) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      // pairs (0,4) (1,5) | (2,6) (3,7) of the lane's 8 k values
      const uint32_t aA[4] = {prmt(a0[u].x, a0[u].z, 0x5410u), prmt(a1[u].x, a1[u].z, 0x5410u),
                              prmt(a0[u].x, a0[u].z, 0x7632u), prmt(a1[u].x, a1[u].z, 0x7632u)};
      const uint32_t aB[4] = {prmt(a0[u].y, a0[u].w, 0x5410u), prmt(a1[u].y, a1[u].w, 0x5410u),
                              prmt(a0[u].y, a0[u].w, 0x7632u), prmt(a1[u].y, a1[u].w, 0x7632u)};
      const uint32_t bA[2] = {prmt(bw[u].x, bw[u].z, 0x5410u), prmt(bw[u].x, bw[u].z, 0x7632u)};
      const uint32_t bB[2] = {prmt(bw[u].y, bw[u].w, 0x5410u), prmt(bw[u].y, bw[u].w, 0x7632u)};
      mma_bf16_16816(acc, aA, bA);
      mma_bf16_16816(acc, aB, bB);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) red[warp][lane][i] = acc[i];
  __syncthreads();
  if (warp == 0) {
    float sum[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w = 0; w < 8; ++w)
#pragma unroll
      for (int i = 0; i < 4; ++i) sum[i] += red[w][lane][i];
    // (token r / r+8, expert 2c / 2c+1)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = t0 + r + 8 * (i >> 1), e = e0 + 2 * c + (i & 1);
      if (t < T) logits[int64_t(t) * E + e] = sum[i] + (bias ? bias[e] : 0.f);
    }
  }
}

// counter (optional): zeroed by the kernel, for the routing kernel after it
static int launch_route_logits(const void* x, int64_t T, int64_t H, const void* wr, const float* bias, int64_t E,
                               float* logits, int32_t* counter, cudaStream_t st) {
  if (E % 8 == 0 && H % 256 == 0) {
    const dim3 g{unsigned(E / 8), unsigned((T + 15) / 16), 1u};
    return launch_kernel(route_logits_mma_kernel, g, dim3{256}, 0, st, static_cast<const __nv_bfloat16*>(x),
                         int(T), int(H), static_cast<const __nv_bfloat16*>(wr), bias, int(E), logits, counter);
  }
  const dim3 g1{unsigned((E + 7) / 8), unsigned((T + RL_TOK - 1) / RL_TOK), 1u};
  const size_t smem = size_t(RL_TOK) * size_t(H) * 2;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(route_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
          cudaSuccess)
    return check_launch();
  return launch_kernel(route_logits_kernel, g1, dim3{256}, smem, st, static_cast<const __nv_bfloat16*>(x), int(T),
                       int(H), static_cast<const __nv_bfloat16*>(wr), bias, int(E), logits, counter);
}

// gates = softmax(logits[t]) (or sigmoid(logits[t]) per expert); top-k by
// gate value (ties -> lower id); scores are the gates of the top-k.  With
// skip > 0 the LExI confidence mask of the reference's skip-fallback forward
// (expert_streaming.py:451-457) follows: slot 0 (the largest gate) is kept,
// slot j >= 1 is zeroed when top1 > skip * score_j.  renorm divides the kept
// scores by their sum when it is positive (:459-460).  One warp per token;
// the E <= 256 logits live in registers (8 per lane).
constexpr int TOPK_PER_LANE = 8;
enum Gating { kGateSoftmax = 0, kGateSigmoid = 1 };

// One warp: gates and top-k of token t's logits.
__device__ __forceinline__ void route_topk_token(float* __restrict__ logits, int t, int E, int k, int renorm,
                                                 int gating, float skip, int32_t* __restrict__ inds,
                                                 float* __restrict__ scores) {
  const int lane = threadIdx.x & 31;
  float* lg = logits + int64_t(t) * E;
  float v[TOPK_PER_LANE];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < TOPK_PER_LANE; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? lg[e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  if (gating == kGateSigmoid) {
#pragma unroll
    for (int i = 0; i < TOPK_PER_LANE; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? 1.f / (1.f + expf(-v[i])) : -1.f;
      if (e < E) lg[e] = v[i];  // leave the gates in the workspace
    }
  } else {
    mx = warp_max<32>(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < TOPK_PER_LANE; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? expf(v[i] - mx) : 0.f;
      sum += v[i];
    }
    sum = warp_sum<32>(sum);
#pragma unroll
    for (int i = 0; i < TOPK_PER_LANE; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? v[i] / sum : -1.f;
      if (e < E) lg[e] = v[i];
    }
  }
  float my_score = 0.f;
  int my_ind = 0;
  for (int j = 0; j < k; ++j) {
    float bv = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < TOPK_PER_LANE; ++i) {
      const int e = lane + 32 * i;
      if (v[i] > bv || (v[i] == bv && e < bi)) {
        bv = v[i];
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
    if (lane == j) {
      my_score = bv;
      my_ind = bi;
    }
    // the owner lane drops the winner from its candidates
    if ((bi & 31) == lane) {
#pragma unroll
      for (int i = 0; i < TOPK_PER_LANE; ++i)
        if (lane + 32 * i == bi) v[i] = -2.f;
    }
  }
  if (skip > 0.f && k > 1) {
    const float top1 = __shfl_sync(0xffffffffu, my_score, 0);
    if (lane > 0 && lane < k && top1 > skip * my_score) my_score = 0.f;
  }
  const float picked = warp_sum<32>(lane < k ? my_score : 0.f);
  if (lane < k) {
    inds[int64_t(t) * k + lane] = my_ind;
    scores[int64_t(t) * k + lane] = (renorm && picked > 0.f) ? my_score / picked : my_score;
  }
}

__global__ void __launch_bounds__(256) route_topk_kernel(float* __restrict__ logits, int T, int E, int k,
                                                         int renorm, int gating, float skip,
                                                         int32_t* __restrict__ inds, float* __restrict__ scores) {
  pdl_enter();
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t < T) route_topk_token(logits, t, E, k, renorm, gating, skip, inds, scores);
}

// Top-k of every token, then -- in the last thread block to finish, found
// with an arrival counter -- the counting sort of the T*k assignments by
// expert (the MoE plan), so routing and planning take one launch.
__global__ void __launch_bounds__(256) route_topk_plan_kernel(float* __restrict__ logits, int T, int E, int k,
                                                              int renorm, int gating, float skip,
                                                              int32_t* __restrict__ inds,
                                                              float* __restrict__ scores, int tile, char* ws,
                                                              PlanLayout L, int32_t* status_out) {
  pdl_enter();
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t < T) route_topk_token(logits, t, E, k, renorm, gating, skip, inds, scores);
  __shared__ int is_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();  // this block's ids visible before it is counted
    int32_t* counter = reinterpret_cast<int32_t*>(ws + L.off_hdr) + 2;
    is_last = atomicAdd(counter, 1) == int(gridDim.x) - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  moe_plan_block(DenseExperts{inds}, T * k, E, tile, ws, L, status_out);
}

// sigmoid of every element (the shared expert's gate logits, [T, E])
__global__ void __launch_bounds__(256) sigmoid_inplace_kernel(float* __restrict__ v, int64_t n) {
  pdl_enter();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    v[i] = 1.f / (1.f + expf(-v[i]));
}

__global__ void __launch_bounds__(1024) argmax_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t V,
                                                           int32_t* __restrict__ out) {
  pdl_enter();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int64_t m = blockIdx.x;
  const __nv_bfloat16* row = x + m * V;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const bool vec = (V % 8) == 0 && (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  if (vec) {
    for (int64_t v = threadIdx.x; v < V / 8; v += blockDim.x) {
      const uint4 q = reinterpret_cast<const uint4*>(row)[v];
      const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = __low2float(q2[i]), b = __high2float(q2[i]);
        if (a > bv) {
          bv = a;
          bi = int(8 * v + 2 * i);
        }
        if (b > bv) {
          bv = b;
          bi = int(8 * v + 2 * i + 1);
        }
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
      const float v = __bfloat162float(row[i]);
      if (v > bv) {
        bv = v;
        bi = int(i);
      }
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

static int qk_norm_rope_impl(const void* qkv, const float* qkv_partial, int nsplit, int64_t B, int64_t Hq,
                             int64_t Hkv, int64_t D, const void* q_norm, const void* k_norm, float eps,
                             float rope_theta, const int32_t* positions, void* q_out, uint8_t* k_codes,
                             float* k_scales, uint8_t* v_codes, float* v_scales, const int32_t* block_table,
                             int64_t max_pages, int64_t page_size, int bits, void* stream) {
  if (D != 128) return B2F_ERR_UNSUPPORTED;
  if (!(bits == 2 || bits == 4 || bits == 8)) return B2F_ERR_UNSUPPORTED;
  if (B < 0 || Hq <= 0 || Hkv <= 0 || page_size <= 0 || max_pages <= 0) return B2F_ERR_INVALID;
  if (B == 0) return B2F_OK;
  if (B > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  if (!q_norm || !k_norm || !positions || !q_out || !k_codes || !k_scales || !v_codes || !v_scales ||
      !block_table)
    return B2F_ERR_INVALID;
  RopeKvParams p{};
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.qkv_partial = qkv_partial;
  p.nsplit = nsplit;
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
  const dim3 grid{unsigned(B), unsigned((Hq + 2 * Hkv + 7) / 8), 1u};
  return launch_kernel(qk_norm_rope_kv_kernel, grid, dim3{256}, 0, as_stream(stream), p);
}

}  // namespace b2f

using namespace b2f;

extern "C" {

int b2f_combine_rmsnorm(const void* resid, const void* y, const float* scores, int64_t M, int64_t k,
                        const void* weight, float eps, int64_t H, void* resid_out, void* norm_out,
                        void* stream) {
  if (M < 0 || H <= 0 || (y && k <= 0)) return B2F_ERR_INVALID;
  if (H % 8 != 0 || H > CMB_CHUNKS * 8 * 256) return B2F_ERR_UNSUPPORTED;
  if (M == 0) return B2F_OK;
  if (!resid || !weight || !norm_out) return B2F_ERR_INVALID;
  if (!aligned(resid, 16) || !aligned(weight, 16) || !aligned(norm_out, 16) || (y && !aligned(y, 16)) ||
      (resid_out && !aligned(resid_out, 16)))
    return B2F_ERR_ALIGN;
  const int threads = int(H / 8) < 256 ? int(((H / 8) + 31) / 32 * 32) : 256;
  return launch_kernel(combine_rmsnorm_kernel, dim3{unsigned(M)}, dim3{unsigned(threads)}, 0, as_stream(stream),
                       static_cast<const __nv_bfloat16*>(resid), static_cast<const __nv_bfloat16*>(y), scores,
                       int(k), static_cast<const __nv_bfloat16*>(weight), eps, int(H),
                       static_cast<__nv_bfloat16*>(resid_out), static_cast<__nv_bfloat16*>(norm_out),
                       static_cast<const float*>(nullptr), 0, int64_t(0));
}

int b2f_combine_rmsnorm_partials(const void* resid, const float* partial, int nsplit, int64_t M,
                                 const void* weight, float eps, int64_t H, void* resid_out, void* norm_out,
                                 void* stream) {
  if (M < 0 || H <= 0 || nsplit < 1) return B2F_ERR_INVALID;
  if (H % 8 != 0 || H > CMB_CHUNKS * 8 * 256) return B2F_ERR_UNSUPPORTED;
  if (M == 0) return B2F_OK;
  if (!resid || !partial || !weight || !norm_out) return B2F_ERR_INVALID;
  if (!aligned(resid, 16) || !aligned(partial, 16) || !aligned(weight, 16) || !aligned(norm_out, 16) ||
      (resid_out && !aligned(resid_out, 16)))
    return B2F_ERR_ALIGN;
  const int threads = int(H / 8) < 256 ? int(((H / 8) + 31) / 32 * 32) : 256;
  return launch_kernel(combine_rmsnorm_kernel, dim3{unsigned(M)}, dim3{unsigned(threads)}, 0, as_stream(stream),
                       static_cast<const __nv_bfloat16*>(resid), static_cast<const __nv_bfloat16*>(nullptr),
                       static_cast<const float*>(nullptr), 0, static_cast<const __nv_bfloat16*>(weight), eps,
                       int(H), static_cast<__nv_bfloat16*>(resid_out), static_cast<__nv_bfloat16*>(norm_out),
                       partial, nsplit, M);
}

int b2f_qk_norm_rope_kv_append_partials(const float* qkv_partial, int nsplit, int64_t B, int64_t Hq, int64_t Hkv,
                                        int64_t D, const void* q_norm, const void* k_norm, float eps,
                                        float rope_theta, const int32_t* positions, void* q_out, uint8_t* k_codes,
                                        float* k_scales, uint8_t* v_codes, float* v_scales,
                                        const int32_t* block_table, int64_t max_pages, int64_t page_size, int bits,
                                        void* stream) {
  if (nsplit < 1 || (!qkv_partial && B > 0)) return B2F_ERR_INVALID;
  return qk_norm_rope_impl(nullptr, qkv_partial, nsplit, B, Hq, Hkv, D, q_norm, k_norm, eps, rope_theta, positions,
                           q_out, k_codes, k_scales, v_codes, v_scales, block_table, max_pages, page_size, bits,
                           stream);
}

int b2f_qk_norm_rope_kv_append(const void* qkv, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                               const void* q_norm, const void* k_norm, float eps, float rope_theta,
                               const int32_t* positions, void* q_out, uint8_t* k_codes, float* k_scales,
                               uint8_t* v_codes, float* v_scales, const int32_t* block_table,
                               int64_t max_pages, int64_t page_size, int bits, void* stream) {
  if (!qkv && B > 0) return B2F_ERR_INVALID;
  return qk_norm_rope_impl(qkv, nullptr, 0, B, Hq, Hkv, D, q_norm, k_norm, eps, rope_theta, positions, q_out,
                           k_codes, k_scales, v_codes, v_scales, block_table, max_pages, page_size, bits, stream);
}

int b2f_moe_route_topk_ex(const void* x, int64_t T, int64_t H, const void* wr, const float* bias, int64_t E,
                          int64_t k, int renorm, int gating, float skip_threshold, float* logits_ws, int32_t* inds,
                          float* scores, void* stream) {
  if (T < 0 || H <= 0 || E <= 0 || k <= 0 || k > E || k > 32) return B2F_ERR_INVALID;
  if (!(gating == kGateSoftmax || gating == kGateSigmoid) || !(skip_threshold >= 0.f)) return B2F_ERR_INVALID;
  if (E > 32 * TOPK_PER_LANE) return B2F_ERR_UNSUPPORTED;
  if (H % 8 != 0) return B2F_ERR_UNSUPPORTED;
  if (T == 0) return B2F_OK;
  if (!x || !wr || !logits_ws || !inds || !scores) return B2F_ERR_INVALID;
  if (!aligned(x, 16) || !aligned(wr, 16)) return B2F_ERR_ALIGN;
  cudaStream_t st = as_stream(stream);
  if (H > 8192) return B2F_ERR_UNSUPPORTED;
  int rc = launch_route_logits(x, T, H, wr, bias, E, logits_ws, nullptr, st);
  if (rc != B2F_OK) return rc;
  return launch_kernel(route_topk_kernel, dim3{unsigned((T + 7) / 8)}, dim3{256}, 0, st, logits_ws, int(T), int(E),
                       int(k), renorm, gating, skip_threshold, inds, scores);
}

int b2f_moe_route_topk(const void* x, int64_t T, int64_t H, const void* wr, const float* bias, int64_t E,
                       int64_t k, int renorm, float* logits_ws, int32_t* inds, float* scores, void* stream) {
  return b2f_moe_route_topk_ex(x, T, H, wr, bias, E, k, renorm, kGateSoftmax, 0.f, logits_ws, inds, scores, stream);
}

int b2f_moe_route_plan_ex(const void* x, int64_t T, int64_t H, const void* wr, const float* bias, int64_t E,
                          int64_t k, int renorm, int gating, float skip_threshold, float* logits_ws, int32_t* inds,
                          float* scores, int tile, void* plan_workspace, int64_t plan_workspace_bytes,
                          int32_t* status_out, void* stream) {
  if (T < 0 || H <= 0 || E <= 0 || k <= 0 || k > E || k > 32) return B2F_ERR_INVALID;
  if (!(gating == kGateSoftmax || gating == kGateSigmoid) || !(skip_threshold >= 0.f)) return B2F_ERR_INVALID;
  if (E > 32 * TOPK_PER_LANE || H % 8 != 0 || H > 8192) return B2F_ERR_UNSUPPORTED;
  if (tile < 8 || tile > 256 || tile % 8 != 0) return B2F_ERR_INVALID;
  if (T * k > 0x3fffffff) return B2F_ERR_UNSUPPORTED;
  if (T == 0) return B2F_OK;
  if (!x || !wr || !logits_ws || !inds || !scores || !plan_workspace) return B2F_ERR_INVALID;
  if (!aligned(x, 16) || !aligned(wr, 16) || !aligned(plan_workspace, 16)) return B2F_ERR_ALIGN;
  const PlanLayout L = plan_layout(T * k, E, tile);
  if (plan_workspace_bytes < L.total) return B2F_ERR_WORKSPACE;
  cudaStream_t st = as_stream(stream);
  char* ws = static_cast<char*>(plan_workspace);
  int rc = launch_route_logits(x, T, H, wr, bias, E, logits_ws, reinterpret_cast<int32_t*>(ws + L.off_hdr) + 2, st);
  if (rc != B2F_OK) return rc;
  return launch_kernel(route_topk_plan_kernel, dim3{unsigned((T + 7) / 8)}, dim3{256}, 0, st, logits_ws, int(T),
                       int(E), int(k), renorm, gating, skip_threshold, inds, scores, tile, ws, L, status_out);
}

int b2f_moe_route_plan(const void* x, int64_t T, int64_t H, const void* wr, const float* bias, int64_t E,
                       int64_t k, int renorm, float* logits_ws, int32_t* inds, float* scores, int tile,
                       void* plan_workspace, int64_t plan_workspace_bytes, int32_t* status_out, void* stream) {
  return b2f_moe_route_plan_ex(x, T, H, wr, bias, E, k, renorm, kGateSoftmax, 0.f, logits_ws, inds, scores, tile,
                               plan_workspace, plan_workspace_bytes, status_out, stream);
}

int b2f_router_logits(const void* x, int64_t T, int64_t H, const void* wr, const float* bias, int64_t E,
                      int apply_sigmoid, float* out, void* stream) {
  if (T < 0 || H <= 0 || E <= 0) return B2F_ERR_INVALID;
  if (E > 32 * TOPK_PER_LANE || H % 8 != 0 || H > 8192) return B2F_ERR_UNSUPPORTED;
  if (T == 0) return B2F_OK;
  if (!x || !wr || !out) return B2F_ERR_INVALID;
  if (!aligned(x, 16) || !aligned(wr, 16)) return B2F_ERR_ALIGN;
  cudaStream_t st = as_stream(stream);
  int rc = launch_route_logits(x, T, H, wr, bias, E, out, nullptr, st);
  if (rc != B2F_OK || !apply_sigmoid) return rc;
  const int64_t n = T * E;
  return launch_kernel(sigmoid_inplace_kernel, dim3{unsigned(n < 148 * 8 * 256 ? (n + 255) / 256 : 148 * 8)},
                       dim3{256}, 0, st, out, n);
}

int b2f_argmax_rows(const void* x, int64_t M, int64_t V, int32_t* out, void* stream) {
  if (M < 0 || V <= 0 || V > 0x7fffffff) return B2F_ERR_INVALID;
  if (M == 0) return B2F_OK;
  if (!x || !out) return B2F_ERR_INVALID;
  return launch_kernel(argmax_rows_kernel, dim3{unsigned(M)}, dim3{1024}, 0, as_stream(stream),
                       static_cast<const __nv_bfloat16*>(x), V, out);
}

}  // extern "C"
