// (a) affine group quantizer/packer, (a') unpacker, (a-kv) reference-format
// symmetric KV quantizer and dequantizer.  All HBM-bound byte/integer work:
// one pass over the input, 16-byte vector loads, warp-shuffle group reductions.
#include <mutex>
#include <string>

#include "common.cuh"

namespace b2f {

static thread_local std::string g_last_error;
void set_last_cuda_error(cudaError_t e) { g_last_error = cudaGetErrorString(e); }

int& launch_pdl_policy() {
  static thread_local int on = 0;
  return on;
}

// ------------------------------------------------------------------------
// (a) affine quantize.  One thread owns EPT consecutive elements of one
// group; TPG = GS/EPT neighbouring lanes reduce min/max with shuffles.
// Two per-group rules, f32 arithmetic with one IEEE rounding per step
// (n = 2^bits - 1):
//   kRuleMlx (mx.quantize): scale = max((max-min)/n, 1e-7); the edge is the
//     larger-magnitude end (min, positive scale, if |min| > |max|; else max
//     with the scale negated); q0 = rint(edge/scale); if q0 != 0 then
//     scale = edge/q0 and bias = edge, else bias = 0; q = clip(rint((w-bias)
//     /scale), 0, n) with the f32 scale and bias, which are rounded into the
//     weight dtype only when stored.
//   kRuleMinMax (the single-linear workload's stated rule): scale =
//     round_T((max-min)/n), bias = min, q = clip(rint((w-min)/scale), 0, n)
//     with the rounded scale; q = 0 for a group whose rounded scale is 0.
// ------------------------------------------------------------------------
enum QuantRule { kRuleMlx = 0, kRuleMinMax = 1 };

// rint(d / s) with d / s the IEEE round-to-nearest quotient, for |d / s| < 2^12.
// d * rcp(s) (rcp correctly rounded) is within 2 ulp of that quotient, so the
// two round to the same integer unless the product lies within 2^-10 of a
// half-integer; only then is the exact division taken.
__device__ __forceinline__ float rint_div(float d, float s, float rs) {
  if (!isfinite(rs)) return rintf(__fdiv_rn(d, s));  // subnormal s: divide exactly
  const float qa = __fmul_rn(d, rs);
  const float fr = fabsf(qa - truncf(qa));
  if (fabsf(fr - 0.5f) < 0.0009765625f) return rintf(__fdiv_rn(d, s));
  return rintf(qa);
}

template <class Tag, int BITS, int GS, int RULE>
__global__ void __launch_bounds__(256) quantize_affine_kernel(const typename Tag::T* __restrict__ w,
                                                              int64_t n_threads,
                                                              uint32_t* __restrict__ wq,
                                                              typename Tag::T* __restrict__ scales,
                                                              typename Tag::T* __restrict__ biases) {
  using T = typename Tag::T;
  constexpr int EPT = (BITS == 2) ? 16 : 8;
  constexpr int TPG = GS / EPT;
  constexpr int WPT = EPT * BITS / 32;
  constexpr int PER = 32 / BITS;
  constexpr float NBINS = float((1 << BITS) - 1);
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t iters = (n_threads + stride - 1) / stride;
  int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int64_t it = 0; it < iters; ++it, t += stride) {
    const bool valid = t < n_threads;
    float v[EPT];
    if (valid) {
      const T* src = w + t * EPT;
      constexpr int VEC = (EPT * int(sizeof(T))) / 16;
      uint4 raw[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) raw[i] = reinterpret_cast<const uint4*>(src)[i];
      const T* vals = reinterpret_cast<const T*>(raw);
#pragma unroll
      for (int i = 0; i < EPT; ++i) v[i] = Tag::to_f(vals[i]);
    } else {
#pragma unroll
      for (int i = 0; i < EPT; ++i) v[i] = 0.f;
    }
    float mx = v[0], mn = v[0];
#pragma unroll
    for (int i = 1; i < EPT; ++i) {
      mx = fmaxf(mx, v[i]);
      mn = fminf(mn, v[i]);
    }
    mx = warp_max<TPG>(mx);
    mn = warp_min<TPG>(mn);
    float scale, bias;
    bool zero_q = false;
    if constexpr (RULE == kRuleMlx) {
      scale = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), NBINS), 1e-7f);
      const bool side = fabsf(mn) > fabsf(mx);
      if (!side) scale = -scale;
      const float edge = side ? mn : mx;
      const float q0 = rintf(__fdiv_rn(edge, scale));
      bias = 0.f;
      if (q0 != 0.f) {
        scale = __fdiv_rn(edge, q0);
        bias = edge;
      }
    } else {
      scale = Tag::round(__fdiv_rn(__fsub_rn(mx, mn), NBINS));
      bias = mn;
      zero_q = scale == 0.f;
    }
    uint32_t words[WPT];
#pragma unroll
    for (int j = 0; j < WPT; ++j) words[j] = 0u;
    const float rs = zero_q ? 0.f : __frcp_rn(scale);
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      uint32_t q = 0u;
      if (!zero_q) {
        float r = rint_div(__fsub_rn(v[i], bias), scale, rs);
        r = fminf(fmaxf(r, 0.f), NBINS);
        q = uint32_t(r);
      }
      words[i / PER] |= q << (BITS * (i % PER));
    }
    if (valid) {
      uint32_t* dst = wq + t * WPT;
      if constexpr (WPT == 2) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(words[0], words[1]);
      } else {
        dst[0] = words[0];
      }
      if ((threadIdx.x % TPG) == 0) {
        const int64_t g = (t * EPT) / GS;
        scales[g] = Tag::from_f(scale);
        biases[g] = Tag::from_f(bias);
      }
    }
  }
}

template <class Tag, int BITS, int RULE>
static int launch_quantize_bits(const void* w, int64_t rows, int64_t K, int gs, uint32_t* wq,
                                void* s, void* b, cudaStream_t st) {
  using T = typename Tag::T;
  constexpr int EPT = (BITS == 2) ? 16 : 8;
  const int64_t n_threads = rows * K / EPT;
  if (n_threads == 0) return B2F_OK;
  const int block = 256;
  int64_t grid = (n_threads + block - 1) / block;
  if (grid > 148 * 64) grid = 148 * 64;
  auto W = static_cast<const T*>(w);
  auto S = static_cast<T*>(s);
  auto Bi = static_cast<T*>(b);
  switch (gs) {
    case 32:
      quantize_affine_kernel<Tag, BITS, 32, RULE><<<grid, block, 0, st>>>(W, n_threads, wq, S, Bi);
      break;
    case 64:
      quantize_affine_kernel<Tag, BITS, 64, RULE><<<grid, block, 0, st>>>(W, n_threads, wq, S, Bi);
      break;
    case 128:
      quantize_affine_kernel<Tag, BITS, 128, RULE><<<grid, block, 0, st>>>(W, n_threads, wq, S, Bi);
      break;
    default:
      return B2F_ERR_UNSUPPORTED;
  }
  return check_launch();
}

template <class Tag, int RULE>
static int launch_quantize(const void* w, int64_t rows, int64_t K, int bits, int gs, uint32_t* wq,
                           void* s, void* b, cudaStream_t st) {
  switch (bits) {
    case 2: return launch_quantize_bits<Tag, 2, RULE>(w, rows, K, gs, wq, s, b, st);
    case 4: return launch_quantize_bits<Tag, 4, RULE>(w, rows, K, gs, wq, s, b, st);
    case 8: return launch_quantize_bits<Tag, 8, RULE>(w, rows, K, gs, wq, s, b, st);
    default: return B2F_ERR_UNSUPPORTED;
  }
}

template <int RULE>
static int quantize_entry(const void* w, int dtype, int64_t rows, int64_t K, int bits, int group_size, uint32_t* wq,
                          void* scales, void* biases, void* stream) {
  if (rows < 0 || K < 0) return B2F_ERR_INVALID;
  if (!(bits == 2 || bits == 4 || bits == 8)) return B2F_ERR_UNSUPPORTED;
  if (!(group_size == 32 || group_size == 64 || group_size == 128)) return B2F_ERR_UNSUPPORTED;
  if (K % group_size != 0) return B2F_ERR_INVALID;
  if (rows * K == 0) return B2F_OK;
  if (!w || !wq || !scales || !biases) return B2F_ERR_INVALID;
  if (!aligned(w, 16) || !aligned(wq, 8)) return B2F_ERR_ALIGN;
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case B2F_BF16: return launch_quantize<TagBF16, RULE>(w, rows, K, bits, group_size, wq, scales, biases, st);
    case B2F_F16: return launch_quantize<TagF16, RULE>(w, rows, K, bits, group_size, wq, scales, biases, st);
    case B2F_F32: return launch_quantize<TagF32, RULE>(w, rows, K, bits, group_size, wq, scales, biases, st);
    default: return B2F_ERR_UNSUPPORTED;
  }
}

// ------------------------------------------------------------------------
// (a') affine dequantize: one thread per 16-byte vector of packed words (4
// words), rows on the grid's y axis; optional row gather.
// w = round_T(q*scale + bias) with an f32 multiply then an f32 add.
// ------------------------------------------------------------------------
template <class Tag, int BITS>
__global__ void __launch_bounds__(256) dequantize_affine_kernel(
    const uint32_t* __restrict__ wq, const typename Tag::T* __restrict__ scales,
    const typename Tag::T* __restrict__ biases, int64_t out_rows, int64_t K, int gs_log2,
    const int32_t* __restrict__ row_index, typename Tag::T* __restrict__ out) {
  pdl_enter();
  using T = typename Tag::T;
  constexpr int PER = 32 / BITS;
  constexpr uint32_t MASK = (1u << BITS) - 1u;
  const int wpr = int(K / PER);
  const int nv = (wpr + 3) / 4;
  const int groups = int(K >> gs_log2);
  // 16-byte word vectors when every row starts 16-byte aligned, else words one by one
  const bool vec = (reinterpret_cast<uintptr_t>(wq) & 15) == 0 && (wpr & 3) == 0;
  for (int64_t r = blockIdx.y; r < out_rows; r += gridDim.y) {
    const int64_t src = row_index ? int64_t(row_index[r]) : r;
    const uint32_t* wrow = wq + src * wpr;
    const T* srow = scales + src * groups;
    const T* brow = biases + src * groups;
    T* orow = out + r * K;
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += gridDim.x * blockDim.x) {
      uint32_t ws[4];
      if (vec) {
        const uint4 w4 = reinterpret_cast<const uint4*>(wrow)[v];
        ws[0] = w4.x;
        ws[1] = w4.y;
        ws[2] = w4.z;
        ws[3] = w4.w;
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u) ws[u] = 4 * v + u < wpr ? wrow[4 * v + u] : 0u;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (4 * v + u >= wpr) break;
        const int k0 = (4 * v + u) * PER;
        const int g = k0 >> gs_log2;
        const float s = Tag::to_f(srow[g]);
        const float b = Tag::to_f(brow[g]);
        T vals[PER];
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          const float q = float((ws[u] >> (BITS * i)) & MASK);
          vals[i] = Tag::from_f(__fadd_rn(__fmul_rn(q, s), b));
        }
        T* dst = orow + k0;
        constexpr int BYTES = PER * int(sizeof(T));
        if constexpr (BYTES % 16 == 0) {
#pragma unroll
          for (int i = 0; i < BYTES / 16; ++i)
            reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(vals)[i];
        } else if constexpr (BYTES == 8) {
          *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(vals);
        } else {
#pragma unroll
          for (int i = 0; i < PER; ++i) dst[i] = vals[i];
        }
      }
    }
  }
}

template <class Tag>
static int launch_dequantize(const uint32_t* wq, const void* s, const void* b, int64_t rows,
                             int64_t K, int bits, int gs, const int32_t* ridx, void* out,
                             cudaStream_t st) {
  using T = typename Tag::T;
  if (rows * K == 0) return B2F_OK;
  const int64_t wpr = K * bits / 32;
  const int64_t nv = (wpr + 3) / 4;
  const int block = nv >= 256 ? 256 : int((nv + 31) / 32 * 32);
  int64_t gx = (nv + block - 1) / block;
  if (gx > 65535) gx = 65535;
  const int64_t gy = rows < 65535 ? rows : 65535;
  const dim3 grid{unsigned(gx), unsigned(gy), 1u};
  const int gl = gs == 32 ? 5 : (gs == 64 ? 6 : 7);
  auto S = static_cast<const T*>(s);
  auto Bi = static_cast<const T*>(b);
  auto O = static_cast<T*>(out);
  auto kern = dequantize_affine_kernel<Tag, 4>;
  switch (bits) {
    case 2: kern = dequantize_affine_kernel<Tag, 2>; break;
    case 4: break;
    case 8: kern = dequantize_affine_kernel<Tag, 8>; break;
    default: return B2F_ERR_UNSUPPORTED;
  }
  return launch_kernel(kern, grid, dim3{unsigned(block)}, 0, st, wq, S, Bi, rows, K, gl, ridx, O);
}

// ------------------------------------------------------------------------
// (a-kv) reference KV quantizer.  One warp per row: per group an absmax
// shuffle reduction, then the codes go to a per-warp shared buffer, then the
// bytes are packed (high nibble first / MSB crumb first).  Each arithmetic
// step rounds into the input dtype exactly like the reference's MLX ops.
// ------------------------------------------------------------------------
struct KvGeom {
  int64_t D, dp, ng, pl;
  int gs, bits, max_int;
};

static KvGeom kv_geom(int64_t D, int bits, int group_size) {
  KvGeom g;
  g.D = D;
  g.gs = int(D < group_size ? D : group_size);
  g.dp = (D % g.gs == 0) ? D : D + g.gs - D % g.gs;
  g.ng = g.dp / g.gs;
  g.pl = bits == 8 ? g.dp : (bits == 4 ? (g.dp + 1) / 2 : (g.dp + 3) / 4);
  g.bits = bits;
  g.max_int = (1 << (bits - 1)) - 1;
  return g;
}

// Fast path of the same quantizer for bf16 rows in whole 64-wide groups (the
// cache's K/V rows, D % 64 == 0): 8 lanes per group, each lane one 16-byte
// load of 8 values, the absmax over the group by shuffles, the codes packed
// in registers and stored as 8 / 4 / 2 bytes.  The per-element arithmetic is
// kv_quantize_kernel's, so the bytes and scales are identical.
template <int BITS>
__global__ void __launch_bounds__(256) kv_quantize_g64_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                              int64_t D, const int64_t* __restrict__ dst_row,
                                                              uint8_t* __restrict__ packed, int64_t packed_ld,
                                                              float* __restrict__ scales, float* __restrict__ zeros,
                                                              int64_t scales_ld) {
  constexpr float MI = float((1 << (BITS - 1)) - 1);
  const int64_t ng = D / 64;
  const int64_t total = rows * ng * 8;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t iters = (total + stride - 1) / stride;
  int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int64_t it = 0; it < iters; ++it, t += stride) {
    const bool valid = t < total;
    const int64_t row = valid ? t / (ng * 8) : 0;
    const int64_t rem = t - row * ng * 8;
    const int64_t grp = rem >> 3;
    const int part = int(rem & 7);
    float v[8];
    if (valid) {
      const uint4 raw = *reinterpret_cast<const uint4*>(x + row * D + grp * 64 + part * 8);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __low2float(h2[i]);
        v[2 * i + 1] = __high2float(h2[i]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
    m = warp_max<8>(m);
    float scale = TagBF16::round(__fdiv_rn(m, MI));
    if (scale == 0.f) scale = 1.f;
    const float rs = __frcp_rn(scale);
    uint32_t c[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // bf16(v / scale): the product with the reciprocal is within 2 ulp of the
      // IEEE quotient, so both round to the same bf16 unless the product's low
      // 16 bits sit within 8 of the bf16 rounding midpoint (then divide exactly)
      float qa = __fmul_rn(v[i], rs);
      const uint32_t lo = __float_as_uint(qa) & 0xFFFFu;
      if (lo - 0x7FF8u <= 0x10u || !isfinite(rs)) qa = __fdiv_rn(v[i], scale);
      const float xs = TagBF16::round(qa);
      float xq = TagBF16::round(rintf(xs));
      xq = fminf(fmaxf(xq, -MI), MI);
      c[i] = uint32_t(int(TagBF16::round(xq + MI)));
    }
    if (!valid) continue;
    const int64_t orow = dst_row ? dst_row[row] : row;
    uint8_t* pr = packed + orow * packed_ld;
    if constexpr (BITS == 8) {
      const uint2 o = make_uint2(c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24),
                                 c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24));
      *reinterpret_cast<uint2*>(pr + grp * 64 + part * 8) = o;
    } else if constexpr (BITS == 4) {
      uint32_t o = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) o |= (((c[2 * i] << 4) | (c[2 * i + 1] & 0xFu)) & 0xFFu) << (8 * i);
      *reinterpret_cast<uint32_t*>(pr + grp * 32 + part * 4) = o;
    } else {
      uint32_t o = 0;
#pragma unroll
      for (int i = 0; i < 2; ++i)
        o |= (((c[4 * i] << 6) | ((c[4 * i + 1] & 3u) << 4) | ((c[4 * i + 2] & 3u) << 2) | (c[4 * i + 3] & 3u)) &
              0xFFu)
             << (8 * i);
      *reinterpret_cast<uint16_t*>(pr + grp * 16 + part * 2) = uint16_t(o);
    }
    if (part == 0) {
      scales[orow * scales_ld + grp] = scale;
      if (zeros) zeros[orow * scales_ld + grp] = 0.f;
    }
  }
}

template <class Tag>
__global__ void kv_quantize_kernel(const typename Tag::T* __restrict__ x, int64_t rows, KvGeom g,
                                   const int64_t* __restrict__ dst_row, uint8_t* __restrict__ packed,
                                   int64_t packed_ld, float* __restrict__ scales,
                                   float* __restrict__ zeros, int64_t scales_ld) {
  extern __shared__ uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int wpb = blockDim.x >> 5;
  const int64_t buf_bytes = (g.dp + 15) & ~int64_t(15);
  uint8_t* codes = smem + warp * buf_bytes;
  const float mi = float(g.max_int);
  for (int64_t row = int64_t(blockIdx.x) * wpb + warp; row < rows; row += int64_t(gridDim.x) * wpb) {
    const typename Tag::T* xr = x + row * g.D;
    const int64_t orow = dst_row ? dst_row[row] : row;
    for (int64_t grp = 0; grp < g.ng; ++grp) {
      const int64_t base = grp * g.gs;
      float m = 0.f;
      for (int j = lane; j < g.gs; j += 32) {
        const int64_t e = base + j;
        const float v = e < g.D ? Tag::to_f(xr[e]) : 0.f;
        m = fmaxf(m, fabsf(v));
      }
      m = warp_max<32>(m);
      float scale = Tag::round(__fdiv_rn(m, mi));
      if (scale == 0.f) scale = 1.f;
      for (int j = lane; j < g.gs; j += 32) {
        const int64_t e = base + j;
        const float v = e < g.D ? Tag::to_f(xr[e]) : 0.f;
        float xs = Tag::round(__fdiv_rn(v, scale));
        float xq = Tag::round(rintf(xs));
        xq = fminf(fmaxf(xq, -mi), mi);
        codes[e] = uint8_t(int(Tag::round(xq + mi)));
      }
      if (lane == 0) {
        scales[orow * scales_ld + grp] = scale;
        if (zeros) zeros[orow * scales_ld + grp] = 0.f;
      }
    }
    __syncwarp();
    uint8_t* pr = packed + orow * packed_ld;
    for (int64_t ob = lane; ob < g.pl; ob += 32) {
      uint8_t byte;
      if (g.bits == 8) {
        byte = codes[ob];
      } else if (g.bits == 4) {
        const int64_t e = 2 * ob;
        const uint8_t c0 = codes[e];
        const uint8_t c1 = (e + 1 < g.dp) ? codes[e + 1] : 0;
        byte = uint8_t((c0 << 4) | (c1 & 0x0F));
      } else {
        const int64_t e = 4 * ob;
        uint8_t c[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i] = (e + i < g.dp) ? codes[e + i] : 0;
        byte = uint8_t((c[0] << 6) | ((c[1] & 3) << 4) | ((c[2] & 3) << 2) | (c[3] & 3));
      }
      pr[ob] = byte;
    }
    __syncwarp();
  }
}

__global__ void kv_dequantize_kernel(const uint8_t* __restrict__ packed, int64_t packed_ld,
                                     const float* __restrict__ scales, int64_t scales_ld,
                                     const int64_t* __restrict__ src_row, int64_t rows, KvGeom g,
                                     float* __restrict__ out) {
  const int64_t n = rows * g.D;
  const float mi = float(g.max_int);
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < n;
       t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = t / g.D, j = t - r * g.D;
    const int64_t sr = src_row ? src_row[r] : r;
    const uint8_t* pr = packed + sr * packed_ld;
    uint32_t code;
    if (g.bits == 8) {
      code = pr[j];
    } else if (g.bits == 4) {
      const uint8_t b = pr[j >> 1];
      code = (j & 1) ? (b & 0x0F) : (b >> 4);
    } else {
      const uint8_t b = pr[j >> 2];
      code = (b >> (6 - 2 * (j & 3))) & 3u;
    }
    out[t] = __fmul_rn(float(code) - mi, scales[sr * scales_ld + j / g.gs]);
  }
}

}  // namespace b2f

using namespace b2f;

extern "C" {

const char* b2f_version(void) { return "b200flash 0.1.0 (sm_100a)"; }

const char* b2f_status_string(int s) {
  switch (s) {
    case B2F_OK: return "ok";
    case B2F_ERR_INVALID: return "invalid argument";
    case B2F_ERR_UNSUPPORTED: return "unsupported bits/group_size/dtype/size";
    case B2F_ERR_ALIGN: return "misaligned pointer or stride";
    case B2F_ERR_CUDA: return "CUDA error";
    case B2F_ERR_TIMEOUT: return "device wait timed out";
    case B2F_ERR_WORKSPACE: return "workspace missing or too small";
    default: return "unknown status";
  }
}

const char* b2f_last_error_string(void) { return g_last_error.c_str(); }

}  // extern "C"

namespace b2f {
int b2f_wait_controls_mma(int op, long long* v);
int b2f_wait_controls_tc(int op, long long* v);
int b2f_wait_controls_tc2(int op, long long* v);
int b2f_wait_controls_gemv(int op, long long* v);
int b2f_wait_controls_attn(int op, long long* v);
int b2f_wait_controls_p2p(int op, long long* v);
static int (*const k_wait_units[])(int, long long*) = {b2f_wait_controls_mma, b2f_wait_controls_tc,
                                                        b2f_wait_controls_tc2, b2f_wait_controls_gemv,
                                                        b2f_wait_controls_attn, b2f_wait_controls_p2p};
}  // namespace b2f

extern "C" {

int b2f_device_status(int32_t* status_out, int clear) {
  if (!status_out) return B2F_ERR_INVALID;
  int32_t st = B2F_OK;
  for (auto f : k_wait_units) {
    long long v = 0;
    if (f(clear ? 1 : 0, &v) != 0) return B2F_ERR_CUDA;
    if (v != 0 && st == B2F_OK) st = int32_t(v);
  }
  *status_out = st;
  return B2F_OK;
}

int b2f_set_wait_limit_ns(int64_t ns) {
  if (ns < 0) return B2F_ERR_INVALID;
  long long v = ns == 0 ? 2000000000ll : (long long)ns;
  for (auto f : k_wait_units)
    if (f(2, &v) != 0) return B2F_ERR_CUDA;
  return B2F_OK;
}

int b2f_set_launch_pdl(int on) {
  const int prev = launch_pdl_policy();
  launch_pdl_policy() = on ? 1 : 0;
  return prev;
}

int b2f_set_producer_stall(int on) {
  long long v = on ? 1 : 0;
  for (auto f : k_wait_units)
    if (f(3, &v) != 0) return B2F_ERR_CUDA;
  return B2F_OK;
}

int b2f_quantize_affine(const void* w, int dtype, int64_t rows, int64_t K, int bits,
                        int group_size, uint32_t* wq, void* scales, void* biases, void* stream) {
  return quantize_entry<kRuleMlx>(w, dtype, rows, K, bits, group_size, wq, scales, biases, stream);
}

int b2f_quantize_affine_minmax(const void* w, int dtype, int64_t rows, int64_t K, int bits, int group_size,
                               uint32_t* wq, void* scales, void* biases, void* stream) {
  return quantize_entry<kRuleMinMax>(w, dtype, rows, K, bits, group_size, wq, scales, biases, stream);
}

int b2f_dequantize_affine(const uint32_t* wq, const void* scales, const void* biases, int dtype,
                          int64_t out_rows, int64_t K, int bits, int group_size,
                          const int32_t* row_index, void* out, void* stream) {
  if (out_rows < 0 || K < 0) return B2F_ERR_INVALID;
  if (!(bits == 2 || bits == 4 || bits == 8)) return B2F_ERR_UNSUPPORTED;
  if (!(group_size == 32 || group_size == 64 || group_size == 128)) return B2F_ERR_UNSUPPORTED;
  if (K % group_size != 0) return B2F_ERR_INVALID;
  if (out_rows * K == 0) return B2F_OK;
  if (!wq || !scales || !biases || !out) return B2F_ERR_INVALID;
  if (!aligned(out, 16)) return B2F_ERR_ALIGN;
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case B2F_BF16: return launch_dequantize<TagBF16>(wq, scales, biases, out_rows, K, bits, group_size, row_index, out, st);
    case B2F_F16: return launch_dequantize<TagF16>(wq, scales, biases, out_rows, K, bits, group_size, row_index, out, st);
    case B2F_F32: return launch_dequantize<TagF32>(wq, scales, biases, out_rows, K, bits, group_size, row_index, out, st);
    default: return B2F_ERR_UNSUPPORTED;
  }
}

int64_t b2f_kv_packed_len(int64_t D, int bits, int group_size) {
  if (D <= 0 || group_size <= 0 || !(bits == 2 || bits == 4 || bits == 8)) return 0;
  return kv_geom(D, bits, group_size).pl;
}

int64_t b2f_kv_num_groups(int64_t D, int group_size) {
  if (D <= 0 || group_size <= 0) return 0;
  return kv_geom(D, 8, group_size).ng;
}

int b2f_kv_quantize_sym(const void* x, int dtype, int64_t rows, int64_t D, int bits,
                        int group_size, const int64_t* dst_row, uint8_t* packed,
                        int64_t packed_ld, float* scales, float* zeros, int64_t scales_ld,
                        void* stream) {
  if (!(bits == 2 || bits == 4 || bits == 8)) return B2F_ERR_UNSUPPORTED;
  if (group_size <= 0 || rows < 0 || D < 0) return B2F_ERR_INVALID;
  if (rows == 0 || D == 0) return B2F_OK;
  if (!x || !packed || !scales) return B2F_ERR_INVALID;
  KvGeom g = kv_geom(D, bits, group_size);
  if (packed_ld < g.pl || scales_ld < g.ng) return B2F_ERR_INVALID;
  const int64_t store_align = bits == 8 ? 8 : (bits == 4 ? 4 : 2);
  if (dtype == B2F_BF16 && g.gs == 64 && D % 64 == 0 && aligned(x, 16) && aligned(packed, 16) &&
      packed_ld % store_align == 0) {
    const int64_t threads = rows * (D / 64) * 8;
    int64_t grid = (threads + 255) / 256;
    if (grid > 148 * 16) grid = 148 * 16;
    cudaStream_t st = as_stream(stream);
    auto xx = static_cast<const __nv_bfloat16*>(x);
    if (bits == 8)
      kv_quantize_g64_kernel<8><<<grid, 256, 0, st>>>(xx, rows, D, dst_row, packed, packed_ld, scales, zeros, scales_ld);
    else if (bits == 4)
      kv_quantize_g64_kernel<4><<<grid, 256, 0, st>>>(xx, rows, D, dst_row, packed, packed_ld, scales, zeros, scales_ld);
    else
      kv_quantize_g64_kernel<2><<<grid, 256, 0, st>>>(xx, rows, D, dst_row, packed, packed_ld, scales, zeros, scales_ld);
    return check_launch();
  }
  const int64_t buf = (g.dp + 15) & ~int64_t(15);
  if (buf > 200 * 1024) return B2F_ERR_UNSUPPORTED;
  int wpb = int(buf <= 48 * 1024 / 8 ? 8 : (48 * 1024 / buf > 0 ? 48 * 1024 / buf : 1));
  const int64_t smem = buf * wpb;
  int64_t grid = (rows + wpb - 1) / wpb;
  if (grid > 148 * 32) grid = 148 * 32;
  cudaStream_t st = as_stream(stream);
  auto launch = [&](auto tag) -> int {
    using Tag = decltype(tag);
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kv_quantize_kernel<Tag>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return B2F_ERR_CUDA;
      }
    }
    kv_quantize_kernel<Tag><<<grid, wpb * 32, smem, st>>>(
        static_cast<const typename Tag::T*>(x), rows, g, dst_row, packed, packed_ld, scales, zeros,
        scales_ld);
    return check_launch();
  };
  switch (dtype) {
    case B2F_BF16: return launch(TagBF16{});
    case B2F_F16: return launch(TagF16{});
    case B2F_F32: return launch(TagF32{});
    default: return B2F_ERR_UNSUPPORTED;
  }
}

int b2f_kv_dequantize_sym(const uint8_t* packed, int64_t packed_ld, const float* scales,
                          int64_t scales_ld, const int64_t* src_row, int64_t rows, int64_t D,
                          int bits, int group_size, float* out, void* stream) {
  if (!(bits == 2 || bits == 4 || bits == 8)) return B2F_ERR_UNSUPPORTED;
  if (group_size <= 0 || rows < 0 || D < 0) return B2F_ERR_INVALID;
  if (rows == 0 || D == 0) return B2F_OK;
  if (!packed || !scales || !out) return B2F_ERR_INVALID;
  KvGeom g = kv_geom(D, bits, group_size);
  if (packed_ld < g.pl || scales_ld < g.ng) return B2F_ERR_INVALID;
  const int64_t n = rows * D;
  int64_t grid = (n + 255) / 256;
  if (grid > 148 * 64) grid = 148 * 64;
  kv_dequantize_kernel<<<grid, 256, 0, as_stream(stream)>>>(packed, packed_ld, scales, scales_ld,
                                                            src_row, rows, g, out);
  return check_launch();
}

}  // extern "C"
