// KV-cache eviction kernels: attention-guided (H2O / ScissorHands,
// kv_compression.py) and sink + window (StreamingLLM, streaming_llm.py).
//
//  * b2f_attn_row_head_mean: the per-token importance of one attention row,
//    mean over heads (kv_compression.py:84-106), written or accumulated
//    (H2O sum :108-127, ScissorHands EMA :129-141) into fp32 score arrays.
//  * b2f_qkv_head_mean_probs: the same importance for the paged quantized
//    decode path, where no attention matrix exists: softmax(q.K^T*scale) of
//    the current query, mean over all query heads, from the packed K pages.
//    Pass 1 (grid B x Hkv x splits) computes per-head (max, sum) partials;
//    pass 2 (grid B x splits) merges them and sums the probabilities of all
//    heads per token.  K is read twice; V is not read.
//  * b2f_evict_keep_indices: the keep list of _compress_layer (:293-364):
//    sink tokens, the `budget - sink - window` most important middle tokens
//    (ties to the lower position) in position order, the recent window.
//    One CTA: radix select of the threshold on order-preserving float keys.
//  * b2f_gather_tokens: dst[o, i, :] = src[o, keep[i], :] for any element
//    size (the reindexing of keys, values and score arrays).
#include "common.cuh"

namespace b2f {

// ---- head mean of an attention row ------------------------------------------
template <class Tag>
__global__ void __launch_bounds__(256) row_head_mean_kernel(const typename Tag::T* __restrict__ attn, int64_t H,
                                                            int64_t head_stride, int64_t S, int mode, float decay,
                                                            float* __restrict__ out, float* __restrict__ out2) {
  for (int64_t s = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; s < S; s += int64_t(gridDim.x) * blockDim.x) {
    float acc = 0.f;
    for (int64_t h = 0; h < H; ++h) acc += Tag::to_f(attn[h * head_stride + s]);
    const float v = acc / float(H);
    if (mode == 0) {
      out[s] = v;
    } else if (mode == 1) {
      out[s] += v;
    } else {
      out[s] = decay * out[s] + (1.0f - decay) * v;
    }
    if (out2) out2[s] += v;
  }
}

// ---- head-mean probabilities over packed K pages ------------------------------
struct HmParams {
  const __nv_bfloat16* q;
  const uint8_t* kp;
  const float* ks;
  const int32_t* block_table;
  int64_t max_pages;
  const int32_t* seq_lens;
  int B, Hq, Hkv, G, D, PS, bits, n_splits, split_len;
  int64_t head_stride, slot_stride;
  float scale;
  float* ml;  // [B][Hq][n_splits][2]
  float* out;
  int64_t out_ld;
  int mode;
  float decay;
};

constexpr int HM_MAXG = 16;  // query heads per KV head handled in registers
constexpr int HM_MAXD = 256;

// score of token t against the G query heads of kv head hkv (one warp)
template <int BITS>
__device__ __forceinline__ void hm_scores(const HmParams& p, int b, int hkv, int t, const float (&qr)[HM_MAXG][HM_MAXD / 32],
                                          float (&sc)[HM_MAXG]) {
  const int lane = threadIdx.x & 31;
  const int page = p.block_table[int64_t(b) * p.max_pages + t / p.PS];
  const int64_t row = int64_t(page) * p.Hkv * p.PS + hkv * p.head_stride + (t % p.PS) * p.slot_stride;
  const int RB = p.D * BITS / 8, DG = p.D / 64;
  const uint8_t* kr = p.kp + row * RB;
  const float* ksr = p.ks + row * DG;
  constexpr float MI = BITS == 8 ? 127.f : BITS == 4 ? 7.f : 1.f;
  float kv[HM_MAXD / 32];
#pragma unroll
  for (int i = 0; i < HM_MAXD / 32; ++i) {
    const int d = lane + 32 * i;
    float v = 0.f;
    if (d < p.D) {
      uint32_t code;
      if constexpr (BITS == 8) {
        code = kr[d];
      } else if constexpr (BITS == 4) {
        const uint8_t byte = kr[d >> 1];
        code = (d & 1) ? (byte & 0xFu) : (byte >> 4);
      } else {
        code = (kr[d >> 2] >> (6 - 2 * (d & 3))) & 0x3u;
      }
      v = (float(code) - MI) * ksr[d >> 6];
    }
    kv[i] = v;
  }
#pragma unroll
  for (int gq = 0; gq < HM_MAXG; ++gq) {
    sc[gq] = -INFINITY;
    if (gq < p.G) {  // p.G is uniform over the warp
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < HM_MAXD / 32; ++i) a = fmaf(qr[gq][i], kv[i], a);
      sc[gq] = warp_sum<32>(a) * p.scale;
    }
  }
}

template <int BITS>
__device__ __forceinline__ void hm_load_q(const HmParams& p, int b, int hkv, float (&qr)[HM_MAXG][HM_MAXD / 32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int gq = 0; gq < HM_MAXG; ++gq)
#pragma unroll
    for (int i = 0; i < HM_MAXD / 32; ++i) {
      const int d = lane + 32 * i;
      qr[gq][i] = (gq < p.G && d < p.D)
                      ? __bfloat162float(p.q[(int64_t(b) * p.Hq + hkv * p.G + gq) * p.D + d])
                      : 0.f;
    }
}

// pass 1: per (sequence, kv head, split) the running max / sum of exp per query head
template <int BITS>
__global__ void __launch_bounds__(128) hm_pass1_kernel(const HmParams p) {
  const int b = blockIdx.z, hkv = blockIdx.y, split = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int len = p.seq_lens[b];
  const int t0 = split * p.split_len, t1 = min(len, t0 + p.split_len);
  float qr[HM_MAXG][HM_MAXD / 32];
  hm_load_q<BITS>(p, b, hkv, qr);
  float m[HM_MAXG], l[HM_MAXG];
#pragma unroll
  for (int g = 0; g < HM_MAXG; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
  }
  for (int t = t0 + warp; t < t1; t += nw) {
    float sc[HM_MAXG];
    hm_scores<BITS>(p, b, hkv, t, qr, sc);
#pragma unroll
    for (int g = 0; g < HM_MAXG; ++g) {
      if (g < p.G) {
        const float mn = fmaxf(m[g], sc[g]);
        l[g] = (l[g] == 0.f ? 0.f : l[g] * __expf(m[g] - mn)) + __expf(sc[g] - mn);
        m[g] = mn;
      }
    }
  }
  __shared__ float sm[4][HM_MAXG][2];
  if (lane == 0)
    for (int g = 0; g < HM_MAXG; ++g) {
      sm[warp][g][0] = m[g];
      sm[warp][g][1] = l[g];
    }
  __syncthreads();
  if (threadIdx.x < p.G) {
    const int g = threadIdx.x;
    float M = -INFINITY, L = 0.f;
    for (int w = 0; w < nw; ++w) {
      const float mw = sm[w][g][0], lw = sm[w][g][1];
      if (lw == 0.f) continue;
      const float mn = fmaxf(M, mw);
      L = (L == 0.f ? 0.f : L * __expf(M - mn)) + lw * __expf(mw - mn);
      M = mn;
    }
    float* dst = p.ml + ((int64_t(b) * p.Hq + hkv * p.G + g) * p.n_splits + split) * 2;
    dst[0] = M;
    dst[1] = L;
  }
}

// pass 2: per (sequence, split) merge the partials and write the head mean
template <int BITS>
__global__ void __launch_bounds__(128) hm_pass2_kernel(const HmParams p) {
  const int b = blockIdx.y, split = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int len = p.seq_lens[b];
  const int t0 = split * p.split_len, t1 = min(len, t0 + p.split_len);
  __shared__ float lse[256];
  for (int h = threadIdx.x; h < p.Hq; h += blockDim.x) {
    const float* src = p.ml + (int64_t(b) * p.Hq + h) * p.n_splits * 2;
    float M = -INFINITY, L = 0.f;
    for (int s = 0; s < p.n_splits; ++s) {
      const float ms = src[2 * s], ls = src[2 * s + 1];
      if (ls == 0.f) continue;
      const float mn = fmaxf(M, ms);
      L = (L == 0.f ? 0.f : L * __expf(M - mn)) + ls * __expf(ms - mn);
      M = mn;
    }
    lse[h] = M + __logf(L);
  }
  __syncthreads();
  float* orow = p.out + int64_t(b) * p.out_ld;
  for (int t = t0 + warp; t < t1; t += nw) {
    float acc = 0.f;
    for (int hkv = 0; hkv < p.Hkv; ++hkv) {
      float qr[HM_MAXG][HM_MAXD / 32];
      hm_load_q<BITS>(p, b, hkv, qr);
      float sc[HM_MAXG];
      hm_scores<BITS>(p, b, hkv, t, qr, sc);
#pragma unroll
      for (int g = 0; g < HM_MAXG; ++g)
        if (g < p.G) acc += __expf(sc[g] - lse[hkv * p.G + g]);
    }
    if (lane == 0) {
      const float v = acc / float(p.Hq);
      if (p.mode == 0) {
        orow[t] = v;
      } else if (p.mode == 1) {
        orow[t] += v;
      } else {
        orow[t] = p.decay * orow[t] + (1.0f - p.decay) * v;
      }
    }
  }
}

// ---- keep list of an attention-guided eviction --------------------------------
__device__ __forceinline__ uint32_t float_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // larger float -> larger key
}

// importance may be NULL: every middle token scores 1 (ties -> position order)
__global__ void __launch_bounds__(1024) keep_indices_kernel(const float* __restrict__ imp, int64_t imp_len, int S,
                                                            int sink, int window, int budget,
                                                            int32_t* __restrict__ keep, int32_t* __restrict__ count) {
  __shared__ int hist[256];
  __shared__ int warp_tot[32];
  __shared__ int total;
  __shared__ uint32_t prefix_s, mask_s;
  __shared__ int need_s;
  const int tid = threadIdx.x;
  const int snk = min(sink, S), win = min(window, S);
  const int mid0 = snk, mid1 = S - win;
  const int mid_len = mid1 - mid0;
  const int mid_budget = max(0, budget - (snk + win));
  const bool evict = S > budget && mid_len > 0 && mid_budget < mid_len;
  if (!evict) {
    for (int i = tid; i < S; i += blockDim.x) keep[i] = i;
    if (tid == 0) *count = S;
    return;
  }
  const bool uniform = imp == nullptr || imp_len < S;
  auto key_of = [&](int t) -> uint32_t { return uniform ? float_key(1.0f) : float_key(imp[t]); };
  // radix select: key of the mid_budget-th largest middle score
  if (tid == 0) {
    prefix_s = 0;
    mask_s = 0;
    need_s = mid_budget;
  }
  __syncthreads();
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = prefix_s, mask = mask_s;
    for (int t = mid0 + tid; t < mid1; t += blockDim.x) {
      const uint32_t k = key_of(t);
      if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 0xFF], 1);
    }
    __syncthreads();
    if (tid == 0) {
      int need = need_s, d = 255;
      for (; d > 0; --d) {
        if (hist[d] >= need) break;
        need -= hist[d];
      }
      need_s = need;
      prefix_s = prefix | (uint32_t(d) << shift);
      mask_s = mask | (0xFFu << shift);
    }
    __syncthreads();
  }
  const uint32_t thr = prefix_s;
  const int ties_needed = need_s;  // how many tokens with key == thr to keep, lowest positions first
  // keep flag per token in position order: sink | (key > thr) or (key == thr and among the first ties) | window
  int tie_run = 0, out_run = 0;
  for (int base = 0; base < S; base += blockDim.x) {
    const int t = base + tid;
    int is_tie = 0;
    uint32_t k = 0;
    if (t >= mid0 && t < mid1) {
      k = key_of(t);
      is_tie = k == thr;
    }
    // exclusive scan of ties
    int v = is_tie, inc = v;
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += n;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      const int nw = blockDim.x >> 5;
      int x = lane < nw ? warp_tot[lane] : 0, xi = x;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, xi, o);
        if (lane >= o) xi += n;
      }
      if (lane < nw) warp_tot[lane] = xi - x;
      if (lane == nw - 1) total = xi;
    }
    __syncthreads();
    const int tie_rank = tie_run + inc - v + warp_tot[warp];
    const int ties_here = total;
    __syncthreads();
    int kf = 0;
    if (t < S) {
      if (t < mid0 || t >= mid1) kf = 1;
      else kf = (k > thr) || (is_tie && tie_rank < ties_needed);
    }
    // exclusive scan of keep flags -> output slot
    inc = kf;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += n;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      const int nw = blockDim.x >> 5;
      int x = lane < nw ? warp_tot[lane] : 0, xi = x;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, xi, o);
        if (lane >= o) xi += n;
      }
      if (lane < nw) warp_tot[lane] = xi - x;
      if (lane == nw - 1) total = xi;
    }
    __syncthreads();
    if (kf) keep[out_run + inc - kf + warp_tot[warp]] = t;
    tie_run += ties_here;
    out_run += total;
    __syncthreads();
  }
  if (tid == 0) *count = out_run;
}

// ---- gather along the token axis --------------------------------------------------
__global__ void __launch_bounds__(256) gather_tokens16_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                              int64_t outer, int64_t S_src, int64_t vecs,
                                                              const int32_t* __restrict__ keep, int64_t n_keep) {
  const int64_t total = outer * n_keep * vecs;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t v = i % vecs, r = i / vecs;
    const int64_t o = r / n_keep, j = r - o * n_keep;
    dst[i] = src[(o * S_src + keep[j]) * vecs + v];
  }
}
__global__ void __launch_bounds__(256) gather_tokens1_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                             int64_t outer, int64_t S_src, int64_t bytes,
                                                             const int32_t* __restrict__ keep, int64_t n_keep) {
  const int64_t total = outer * n_keep * bytes;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t v = i % bytes, r = i / bytes;
    const int64_t o = r / n_keep, j = r - o * n_keep;
    dst[i] = src[(o * S_src + keep[j]) * bytes + v];
  }
}

static int grid_cap(int64_t n) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n + 255) / 256;
  return int(want < 1 ? 1 : (want > int64_t(sms) * 8 ? int64_t(sms) * 8 : want));
}

}  // namespace b2f

using namespace b2f;

extern "C" {

int b2f_attn_row_head_mean(const void* attn, int dtype, int64_t H, int64_t head_stride, int64_t S, int mode,
                           float decay, float* out, float* out2, void* stream) {
  if (H <= 0 || S < 0 || head_stride < S || mode < 0 || mode > 2) return B2F_ERR_INVALID;
  if (S == 0) return B2F_OK;
  if (!attn || !out) return B2F_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  const int grid = grid_cap(S);
  if (dtype == B2F_BF16)
    row_head_mean_kernel<TagBF16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(attn), H, head_stride, S,
                                                        mode, decay, out, out2);
  else if (dtype == B2F_F16)
    row_head_mean_kernel<TagF16><<<grid, 256, 0, st>>>(static_cast<const __half*>(attn), H, head_stride, S, mode,
                                                       decay, out, out2);
  else if (dtype == B2F_F32)
    row_head_mean_kernel<TagF32><<<grid, 256, 0, st>>>(static_cast<const float*>(attn), H, head_stride, S, mode,
                                                       decay, out, out2);
  else
    return B2F_ERR_UNSUPPORTED;
  return check_launch();
}

int64_t b2f_qkv_head_mean_probs_workspace_bytes(int64_t B, int64_t Hq, int n_splits) {
  if (B <= 0 || Hq <= 0 || n_splits <= 0) return 0;
  return B * Hq * n_splits * 2 * int64_t(sizeof(float));
}

int b2f_qkv_head_mean_probs(const void* q, const uint8_t* k_pages, const float* k_scales, const int32_t* block_table,
                            int64_t max_pages, const int32_t* seq_lens, int64_t max_len, int64_t B, int64_t Hq,
                            int64_t Hkv, int64_t D, int64_t page_size, int64_t head_stride, int64_t slot_stride,
                            int bits, int group_size, float softmax_scale, int n_splits, void* workspace,
                            int64_t workspace_bytes, float* out, int64_t out_ld, int mode, float decay, void* stream) {
  if (!(bits == 2 || bits == 4 || bits == 8)) return B2F_ERR_UNSUPPORTED;
  if (group_size != 64 || D % 64 != 0 || D > HM_MAXD) return B2F_ERR_UNSUPPORTED;
  if (B < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || Hq / Hkv > HM_MAXG || Hq > 256) return B2F_ERR_UNSUPPORTED;
  if (page_size <= 0 || max_pages <= 0 || max_len < 0 || out_ld < max_len || n_splits <= 0 || mode < 0 || mode > 2)
    return B2F_ERR_INVALID;
  if (B == 0 || max_len == 0) return B2F_OK;
  if (!q || !k_pages || !k_scales || !block_table || !seq_lens || !out) return B2F_ERR_INVALID;
  const int64_t need = b2f_qkv_head_mean_probs_workspace_bytes(B, Hq, n_splits);
  if (!workspace || workspace_bytes < need) return B2F_ERR_WORKSPACE;
  if (B > 65535 || Hkv > 65535) return B2F_ERR_UNSUPPORTED;
  HmParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.kp = k_pages;
  p.ks = k_scales;
  p.block_table = block_table;
  p.max_pages = max_pages;
  p.seq_lens = seq_lens;
  p.B = int(B);
  p.Hq = int(Hq);
  p.Hkv = int(Hkv);
  p.G = int(Hq / Hkv);
  p.D = int(D);
  p.PS = int(page_size);
  p.bits = bits;
  p.n_splits = n_splits;
  p.split_len = int((max_len + n_splits - 1) / n_splits);
  p.head_stride = head_stride;
  p.slot_stride = slot_stride;
  p.scale = softmax_scale;
  p.ml = static_cast<float*>(workspace);
  p.out = out;
  p.out_ld = out_ld;
  p.mode = mode;
  p.decay = decay;
  cudaStream_t st = as_stream(stream);
  const dim3 g1{unsigned(n_splits), unsigned(Hkv), unsigned(B)};
  const dim3 g2{unsigned(n_splits), unsigned(B), 1u};
  if (bits == 8) {
    hm_pass1_kernel<8><<<g1, 128, 0, st>>>(p);
    hm_pass2_kernel<8><<<g2, 128, 0, st>>>(p);
  } else if (bits == 2) {
    hm_pass1_kernel<2><<<g1, 128, 0, st>>>(p);
    hm_pass2_kernel<2><<<g2, 128, 0, st>>>(p);
  } else {
    hm_pass1_kernel<4><<<g1, 128, 0, st>>>(p);
    hm_pass2_kernel<4><<<g2, 128, 0, st>>>(p);
  }
  return check_launch();
}

int b2f_evict_keep_indices(const float* importance, int64_t importance_len, int64_t S, int64_t sink,
                           int64_t window, int64_t budget, int32_t* keep, int32_t* count, void* stream) {
  if (S < 0 || sink < 0 || window < 0 || budget < 0 || importance_len < 0) return B2F_ERR_INVALID;
  if (S > 0x3fffffff) return B2F_ERR_UNSUPPORTED;
  if (!keep || !count) return B2F_ERR_INVALID;
  keep_indices_kernel<<<1, 1024, 0, as_stream(stream)>>>(importance, importance_len, int(S),
                                                         int(sink < S ? sink : S), int(window < S ? window : S),
                                                         int(budget < S ? budget : S), keep, count);
  return check_launch();
}

int b2f_gather_tokens(const void* src, void* dst, int64_t outer, int64_t S_src, int64_t row_bytes,
                      const int32_t* keep, int64_t n_keep, void* stream) {
  if (outer < 0 || S_src < 0 || row_bytes <= 0 || n_keep < 0) return B2F_ERR_INVALID;
  if (outer == 0 || n_keep == 0) return B2F_OK;
  if (!src || !dst || !keep) return B2F_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (row_bytes % 16 == 0 && aligned(src, 16) && aligned(dst, 16)) {
    const int64_t vecs = row_bytes / 16;
    gather_tokens16_kernel<<<grid_cap(outer * n_keep * vecs), 256, 0, st>>>(
        static_cast<const uint4*>(src), static_cast<uint4*>(dst), outer, S_src, vecs, keep, n_keep);
  } else {
    gather_tokens1_kernel<<<grid_cap(outer * n_keep * row_bytes), 256, 0, st>>>(
        static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), outer, S_src, row_bytes, keep, n_keep);
  }
  return check_launch();
}

}  // extern "C"

// ---- compaction of a paged quantized cache ----------------------------------
// For sequence b and kept position i < n_keep[b]: token keep[b][i] of the
// source pages (block table bt_src) moves to position i of the destination
// pages (bt_dst), for every KV head: codes (RB bytes) and scales (DG floats)
// of K and V.  Head-major pages [page][Hkv][PS]; one warp per (b, i, head).
namespace b2f {
__global__ void __launch_bounds__(256) kv_pages_gather_kernel(
    const uint8_t* __restrict__ kp, const float* __restrict__ ks, const uint8_t* __restrict__ vp,
    const float* __restrict__ vs, const int32_t* __restrict__ bt_src, const int32_t* __restrict__ keep,
    int64_t keep_ld, const int32_t* __restrict__ n_keep, uint8_t* __restrict__ kp_out, float* __restrict__ ks_out,
    uint8_t* __restrict__ vp_out, float* __restrict__ vs_out, const int32_t* __restrict__ bt_dst, int64_t max_pages,
    int B, int Hkv, int PS, int RB, int DG, int64_t max_keep) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t total = int64_t(B) * max_keep * Hkv;
  if (wid >= total) return;
  const int h = int(wid % Hkv);
  const int64_t rest = wid / Hkv;
  const int64_t i = rest % max_keep;
  const int b = int(rest / max_keep);
  if (i >= n_keep[b]) return;
  const int t = keep[int64_t(b) * keep_ld + i];
  if (t < 0 || t / PS >= max_pages || i / PS >= max_pages) return;  // keep entry outside the block table
  const int64_t src = (int64_t(bt_src[int64_t(b) * max_pages + t / PS]) * Hkv + h) * PS + t % PS;
  const int64_t dst = (int64_t(bt_dst[int64_t(b) * max_pages + i / PS]) * Hkv + h) * PS + i % PS;
  for (int o = lane * 4; o < RB; o += 128) {
    *reinterpret_cast<uint32_t*>(kp_out + dst * RB + o) = *reinterpret_cast<const uint32_t*>(kp + src * RB + o);
    *reinterpret_cast<uint32_t*>(vp_out + dst * RB + o) = *reinterpret_cast<const uint32_t*>(vp + src * RB + o);
  }
  if (lane < DG) {
    ks_out[dst * DG + lane] = ks[src * DG + lane];
    vs_out[dst * DG + lane] = vs[src * DG + lane];
  }
}
}  // namespace b2f

extern "C" int b2f_kv_pages_gather(const uint8_t* k_pages, const float* k_scales, const uint8_t* v_pages,
                                   const float* v_scales, const int32_t* block_table_src, const int32_t* keep,
                                   int64_t keep_ld, const int32_t* n_keep, int64_t max_keep, uint8_t* k_pages_out,
                                   float* k_scales_out, uint8_t* v_pages_out, float* v_scales_out,
                                   const int32_t* block_table_dst, int64_t max_pages, int64_t B, int64_t Hkv,
                                   int64_t D, int64_t page_size, int bits, void* stream) {
  if (!(bits == 2 || bits == 4 || bits == 8)) return B2F_ERR_UNSUPPORTED;
  if (B < 0 || Hkv <= 0 || D <= 0 || D % 64 != 0 || page_size <= 0 || max_pages <= 0 || max_keep < 0 ||
      keep_ld < max_keep)
    return B2F_ERR_INVALID;
  const int RB = int(D * bits / 8);
  if (RB % 4 != 0) return B2F_ERR_UNSUPPORTED;
  if (B == 0 || max_keep == 0) return B2F_OK;
  if (!k_pages || !k_scales || !v_pages || !v_scales || !block_table_src || !keep || !n_keep || !k_pages_out ||
      !k_scales_out || !v_pages_out || !v_scales_out || !block_table_dst)
    return B2F_ERR_INVALID;
  if (!aligned(k_pages, 4) || !aligned(v_pages, 4) || !aligned(k_pages_out, 4) || !aligned(v_pages_out, 4))
    return B2F_ERR_ALIGN;
  const int64_t warps = B * max_keep * Hkv;
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  kv_pages_gather_kernel<<<unsigned(blocks), 256, 0, as_stream(stream)>>>(
      k_pages, k_scales, v_pages, v_scales, block_table_src, keep, keep_ld, n_keep, k_pages_out, k_scales_out,
      v_pages_out, v_scales_out, block_table_dst, max_pages, int(B), int(Hkv), int(page_size), RB, int(D / 64),
      max_keep);
  return check_launch();
}
