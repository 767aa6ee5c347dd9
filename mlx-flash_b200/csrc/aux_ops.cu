// Smaller kernels around the quantized hot path:
//
//  * Q4_0 dequant-GEMV: the Metal `flash_dequant_gemv_q4` shader's format
//    (kernels/flash_dequant.metal:19-49): uint8 codes, two per byte, low
//    nibble first, value (code - 8) * scale, one fp16 scale per group, fp32
//    input and output vectors.
//  * The two standalone ops of kernels/ops.py: SwiGLU (:48-108) and the
//    top-k weighted expert sum `moe_dispatch` (:111-148).  The decode step
//    fuses both into other kernels; these are the drop-in forms.
//  * 4-bit -> 2-bit expert requantization and 2-bit dequantization
//    (mixed_precision.py:130-255), bit-exact with the NumPy reference.
//  * Per-tensor symmetric fake quantization for layer-sensitivity scoring
//    (layer_quantization.py:461-494).
#include "common.cuh"

namespace b2f {

// ---- Q4_0 GEMV ------------------------------------------------------------
// y[b, m] = sum_n (code(m, n) - 8) * scale(m, n / gs) * x[b, n]
// A warp owns Q4_ROWS consecutive rows; x is staged in shared memory in
// chunks of Q4_NC elements for up to Q4_VEC vectors at a time.  Lane l takes
// the 16-byte (32-code) pieces l, l+32, ... of the chunk for every row it
// owns, so one shared-memory read of x serves Q4_ROWS rows.
constexpr int Q4_ROWS = 4;
constexpr int Q4_WARPS = 8;
constexpr int Q4_NC = 2048;
constexpr int Q4_VEC = 2;

__global__ void __launch_bounds__(Q4_WARPS * 32) q4_0_gemv_kernel(const uint8_t* __restrict__ w,
                                                                  const __half* __restrict__ scales,
                                                                  const float* __restrict__ x, float* __restrict__ y,
                                                                  int64_t M, int64_t N, int gs, int64_t nvec) {
  __shared__ __align__(16) float xs[Q4_VEC][Q4_NC];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row0 = (int64_t(blockIdx.x) * Q4_WARPS + warp) * Q4_ROWS;
  const int64_t ng = N / gs;
  for (int64_t b0 = 0; b0 < nvec; b0 += Q4_VEC) {
    const int nb = int(nvec - b0 < Q4_VEC ? nvec - b0 : Q4_VEC);
    float acc[Q4_ROWS][Q4_VEC];
#pragma unroll
    for (int r = 0; r < Q4_ROWS; ++r)
#pragma unroll
      for (int v = 0; v < Q4_VEC; ++v) acc[r][v] = 0.f;
    for (int64_t n0 = 0; n0 < N; n0 += Q4_NC) {
      const int nc = int(N - n0 < Q4_NC ? N - n0 : Q4_NC);
      __syncthreads();
      for (int v = 0; v < nb; ++v)
        for (int i = threadIdx.x; i < nc; i += blockDim.x) xs[v][i] = x[(b0 + v) * N + n0 + i];
      __syncthreads();
      for (int piece = lane; piece * 32 < nc; piece += 32) {
        const int64_t col = n0 + int64_t(piece) * 32;  // first code of this piece
        uint4 wv[Q4_ROWS];
        float sc[Q4_ROWS];
#pragma unroll
        for (int r = 0; r < Q4_ROWS; ++r) {
          const int64_t m = row0 + r;
          if (m < M) {
            wv[r] = *reinterpret_cast<const uint4*>(w + m * (N / 2) + col / 2);
            sc[r] = __half2float(scales[m * ng + col / gs]);
          } else {
            wv[r] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
            sc[r] = 0.f;
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
#pragma unroll
          for (int h = 0; h < 8; ++h) {
            const int i = q * 8 + h;  // code index inside the piece
            float xv[Q4_VEC];
#pragma unroll
            for (int v = 0; v < Q4_VEC; ++v) xv[v] = v < nb ? xs[v][piece * 32 + i] : 0.f;
#pragma unroll
            for (int r = 0; r < Q4_ROWS; ++r) {
              const uint32_t word = q == 0 ? wv[r].x : q == 1 ? wv[r].y : q == 2 ? wv[r].z : wv[r].w;
              // byte h/2 of the word; low nibble = even code, high nibble = odd code
              const uint32_t code = (word >> (4 * h)) & 0xFu;
              const float wvf = (float(int(code)) - 8.0f) * sc[r];
#pragma unroll
              for (int v = 0; v < Q4_VEC; ++v) acc[r][v] = fmaf(wvf, xv[v], acc[r][v]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < Q4_ROWS; ++r)
#pragma unroll
      for (int v = 0; v < Q4_VEC; ++v) {
        const float s = warp_sum<32>(acc[r][v]);
        const int64_t m = row0 + r;
        if (lane == 0 && m < M && v < nb) y[(b0 + v) * M + m] = s;
      }
  }
}

// ---- SwiGLU and the weighted expert sum ----------------------------------
template <class Tag>
__global__ void __launch_bounds__(256) swiglu_kernel(const typename Tag::T* __restrict__ gate,
                                                     const typename Tag::T* __restrict__ up,
                                                     typename Tag::T* __restrict__ out, int64_t n) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const float g = Tag::to_f(gate[i]);
    const float u = Tag::to_f(up[i]);
    out[i] = Tag::from_f(g / (1.0f + expf(-g)) * u);
  }
}

// out[t, h] = sum_j expert_outputs[t][ids[t, j], h] * weights[t, j]  (fp32 sum)
template <class Tag>
__global__ void __launch_bounds__(256) moe_dispatch_kernel(const typename Tag::T* __restrict__ eo,
                                                           int64_t eo_token_stride, int64_t H,
                                                           const int32_t* __restrict__ ids,
                                                           const float* __restrict__ wts, int k,
                                                           typename Tag::T* __restrict__ out) {
  const int64_t t = blockIdx.y;
  const typename Tag::T* base = eo + t * eo_token_stride;
  for (int64_t h = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; h < H; h += int64_t(gridDim.x) * blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc += Tag::to_f(base[int64_t(ids[t * k + j]) * H + h]) * wts[t * k + j];
    out[t * H + h] = Tag::from_f(acc);
  }
}

// ---- 4-bit -> 2-bit requantization ---------------------------------------
// One lane segment of LPG = wpg / VPL lanes per (row, group); a lane holds
// VPL consecutive codes (VPL/2 source bytes, VPL/4 output bytes).  All float
// steps are separately rounded fp32 ops, as NumPy evaluates them:
//   v = nib * s + b;  range = max - min (1e-10 if below);
//   crumb = clip(rint((v - min) / range * 3), 0, 3);
//   scale2 = fp16(range / 3), bias2 = fp16(min).
template <class Tag, int VPL>
__global__ void __launch_bounds__(256) requant_4to2_kernel(const uint32_t* __restrict__ wq, int64_t rows,
                                                           int64_t cols_u32, const typename Tag::T* __restrict__ s,
                                                           const typename Tag::T* __restrict__ b, int64_t ng,
                                                           int wpg, uint8_t* __restrict__ packed,
                                                           __half* __restrict__ s2, __half* __restrict__ b2) {
  const int lpg = wpg / VPL;  // power of two, <= 32
  const int64_t seg = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / lpg;  // (row, group) id
  const int sl = threadIdx.x & (lpg - 1);
  const bool live = seg < rows * ng;
  const int64_t row = live ? seg / ng : 0, g = live ? seg % ng : 0;
  float v[VPL];
  float mn = 3.402823466e38f, mx = -3.402823466e38f;
  if (live) {
    const float sc = Tag::to_f(s[row * ng + g]);
    const float bi = Tag::to_f(b[row * ng + g]);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(wq + row * cols_u32);
    const int64_t c0 = g * wpg + int64_t(sl) * VPL;  // first code of this lane
#pragma unroll
    for (int i = 0; i < VPL; i += 2) {
      const uint8_t byte = src[(c0 + i) / 2];
      v[i] = __fadd_rn(__fmul_rn(float(byte & 0xF), sc), bi);
      v[i + 1] = __fadd_rn(__fmul_rn(float(byte >> 4), sc), bi);
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      mn = fminf(mn, v[i]);
      mx = fmaxf(mx, v[i]);
    }
  }
  for (int o = lpg / 2; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (!live) return;
  float range = __fsub_rn(mx, mn);
  if (range < 1e-10f) range = 1e-10f;
  uint8_t* dst = packed + row * (cols_u32 * 2) + (g * wpg + int64_t(sl) * VPL) / 4;
#pragma unroll
  for (int i = 0; i < VPL; i += 4) {
    uint32_t byte = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float c = rintf(__fmul_rn(__fdiv_rn(__fsub_rn(v[i + j], mn), range), 3.0f));
      c = fminf(fmaxf(c, 0.f), 3.f);
      byte |= uint32_t(c) << (2 * j);
    }
    dst[i / 4] = uint8_t(byte);
  }
  if (sl == 0) {
    s2[row * ng + g] = __float2half_rn(__fdiv_rn(range, 3.0f));
    b2[row * ng + g] = __float2half_rn(mn);
  }
}

// out[r, j] = crumb(r, j) * scale2 + bias2 (fp32; fp16 scale/bias widened)
__global__ void __launch_bounds__(256) dequant_2bit_kernel(const uint8_t* __restrict__ packed, int64_t packed_ld,
                                                           const __half* __restrict__ s2,
                                                           const __half* __restrict__ b2, int64_t ng, int64_t rows,
                                                           int64_t n, float* __restrict__ out) {
  const int64_t wpg = n / ng;
  const int64_t total = rows * n;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / n, j = i - r * n;
    const uint32_t c = (packed[r * packed_ld + j / 4] >> (2 * (j % 4))) & 3u;
    const int64_t g = j / wpg;
    out[i] = __fadd_rn(__fmul_rn(float(c), __half2float(s2[r * ng + g])), __half2float(b2[r * ng + g]));
  }
}

// ---- per-tensor symmetric fake quantization ------------------------------
// absmax of |w| (non-negative floats order like their bit patterns)
template <class Tag>
__global__ void __launch_bounds__(256) absmax_kernel(const typename Tag::T* __restrict__ w, int64_t n,
                                                     unsigned int* __restrict__ out_bits) {
  float m = 0.f;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(Tag::to_f(w[i])));
  m = warp_max<32>(m);
  __shared__ float sh[8];
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < int(blockDim.x >> 5); ++i) t = fmaxf(t, sh[i]);
    atomicMax(out_bits, __float_as_uint(t));
  }
}

// scale = max(dtype(absmax / qmax), 1e-10) in fp32 (the 1e-10 floor is an
// fp32 array, which promotes the result); out = clip(rint(w / scale),
// qmin, qmax) * scale in fp32.
template <class Tag>
__global__ void __launch_bounds__(256) fake_quant_kernel(const typename Tag::T* __restrict__ w, int64_t n,
                                                         const unsigned int* __restrict__ absmax_bits, float qmin,
                                                         float qmax, float* __restrict__ out) {
  const float amax = __uint_as_float(*absmax_bits);
  const float scale = fmaxf(Tag::round(__fdiv_rn(amax, qmax)), 1e-10f);
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    float q = rintf(__fdiv_rn(Tag::to_f(w[i]), scale));
    q = fminf(fmaxf(q, qmin), qmax);
    out[i] = __fmul_rn(q, scale);
  }
}

static int grid_for(int64_t n, int threads) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n + threads - 1) / threads;
  const int64_t cap = int64_t(sms) * 8;
  return int(want < 1 ? 1 : (want > cap ? cap : want));
}

template <int VPL, class Tag>
static void launch_requant(const uint32_t* wq, int64_t rows, int64_t cols_u32, const void* s, const void* b,
                           int64_t ng, int wpg, uint8_t* packed, __half* s2, __half* b2, cudaStream_t st) {
  const int lpg = wpg / VPL;
  const int64_t threads_total = rows * ng * lpg;
  const int64_t blocks = (threads_total + 255) / 256;
  requant_4to2_kernel<Tag, VPL><<<unsigned(blocks), 256, 0, st>>>(
      wq, rows, cols_u32, static_cast<const typename Tag::T*>(s), static_cast<const typename Tag::T*>(b), ng, wpg,
      packed, s2, b2);
}

template <class Tag>
static int requant_dispatch(const uint32_t* wq, int64_t rows, int64_t cols_u32, const void* s, const void* b,
                            int64_t ng, int wpg, uint8_t* packed, __half* s2, __half* b2, cudaStream_t st) {
  // lanes per group <= 32; at least 4 codes (one output byte) per lane
  if (wpg <= 128) {
    launch_requant<4, Tag>(wq, rows, cols_u32, s, b, ng, wpg, packed, s2, b2, st);
  } else if (wpg == 256) {
    launch_requant<8, Tag>(wq, rows, cols_u32, s, b, ng, wpg, packed, s2, b2, st);
  } else if (wpg == 512) {
    launch_requant<16, Tag>(wq, rows, cols_u32, s, b, ng, wpg, packed, s2, b2, st);
  } else if (wpg == 1024) {
    launch_requant<32, Tag>(wq, rows, cols_u32, s, b, ng, wpg, packed, s2, b2, st);
  } else {
    return B2F_ERR_UNSUPPORTED;
  }
  return check_launch();
}

}  // namespace b2f

using namespace b2f;

extern "C" {

int b2f_q4_0_gemv(const uint8_t* weights, const void* scales, const float* x, float* y, int64_t M, int64_t N,
                  int group_size, int64_t nvec, void* stream) {
  if (M < 0 || N < 0 || nvec < 0) return B2F_ERR_INVALID;
  if (group_size <= 0 || group_size % 32 != 0) return B2F_ERR_UNSUPPORTED;
  if (N % group_size != 0) return B2F_ERR_INVALID;
  if (M == 0 || nvec == 0) return B2F_OK;
  if (N == 0) return B2F_ERR_INVALID;
  if (!weights || !scales || !x || !y) return B2F_ERR_INVALID;
  if (!aligned(weights, 16) || !aligned(scales, 2) || !aligned(x, 4) || !aligned(y, 4)) return B2F_ERR_ALIGN;
  const int64_t blocks = (M + Q4_WARPS * Q4_ROWS - 1) / (Q4_WARPS * Q4_ROWS);
  if (blocks > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  q4_0_gemv_kernel<<<unsigned(blocks), Q4_WARPS * 32, 0, as_stream(stream)>>>(
      weights, static_cast<const __half*>(scales), x, y, M, N, group_size, nvec);
  return check_launch();
}

int b2f_swiglu(const void* gate, const void* up, void* out, int64_t n, int dtype, void* stream) {
  if (n < 0) return B2F_ERR_INVALID;
  if (n == 0) return B2F_OK;
  if (!gate || !up || !out) return B2F_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  const int grid = grid_for(n, 256);
  if (dtype == B2F_BF16)
    swiglu_kernel<TagBF16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(gate),
                                                 static_cast<const __nv_bfloat16*>(up),
                                                 static_cast<__nv_bfloat16*>(out), n);
  else if (dtype == B2F_F16)
    swiglu_kernel<TagF16><<<grid, 256, 0, st>>>(static_cast<const __half*>(gate), static_cast<const __half*>(up),
                                                static_cast<__half*>(out), n);
  else if (dtype == B2F_F32)
    swiglu_kernel<TagF32><<<grid, 256, 0, st>>>(static_cast<const float*>(gate), static_cast<const float*>(up),
                                                static_cast<float*>(out), n);
  else
    return B2F_ERR_UNSUPPORTED;
  return check_launch();
}

int b2f_moe_dispatch(const void* expert_outputs, int64_t eo_token_stride, int64_t E, int64_t H,
                     const int32_t* selected_ids, const float* routing_weights, int64_t T, int64_t k, int dtype,
                     void* out, void* stream) {
  if (E <= 0 || H < 0 || T < 0 || k <= 0 || eo_token_stride < 0) return B2F_ERR_INVALID;
  if (T == 0 || H == 0) return B2F_OK;
  if (!expert_outputs || !selected_ids || !routing_weights || !out) return B2F_ERR_INVALID;
  if (T > 65535) return B2F_ERR_UNSUPPORTED;
  cudaStream_t st = as_stream(stream);
  const dim3 grid{unsigned((H + 255) / 256 < 1024 ? (H + 255) / 256 : 1024), unsigned(T)};
  if (dtype == B2F_BF16)
    moe_dispatch_kernel<TagBF16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(expert_outputs),
                                                       eo_token_stride, H, selected_ids, routing_weights, int(k),
                                                       static_cast<__nv_bfloat16*>(out));
  else if (dtype == B2F_F16)
    moe_dispatch_kernel<TagF16><<<grid, 256, 0, st>>>(static_cast<const __half*>(expert_outputs), eo_token_stride,
                                                      H, selected_ids, routing_weights, int(k),
                                                      static_cast<__half*>(out));
  else if (dtype == B2F_F32)
    moe_dispatch_kernel<TagF32><<<grid, 256, 0, st>>>(static_cast<const float*>(expert_outputs), eo_token_stride,
                                                      H, selected_ids, routing_weights, int(k),
                                                      static_cast<float*>(out));
  else
    return B2F_ERR_UNSUPPORTED;
  return check_launch();
}

int b2f_requant_4to2(const uint32_t* wq, int64_t rows, int64_t cols_u32, const void* scales, const void* biases,
                     int dtype, int64_t n_groups, uint8_t* packed, void* scales2, void* biases2, void* stream) {
  if (rows < 0 || cols_u32 <= 0 || n_groups <= 0) return B2F_ERR_INVALID;
  const int64_t n = cols_u32 * 8;
  if (n % n_groups != 0) return B2F_ERR_INVALID;
  const int64_t wpg = n / n_groups;
  if (wpg < 4 || wpg > 1024 || (wpg & (wpg - 1)) != 0) return B2F_ERR_UNSUPPORTED;
  if (rows == 0) return B2F_OK;
  if (!wq || !scales || !biases || !packed || !scales2 || !biases2) return B2F_ERR_INVALID;
  if (rows * n_groups * (wpg / 4) / 256 > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  cudaStream_t st = as_stream(stream);
  __half* s2 = static_cast<__half*>(scales2);
  __half* b2 = static_cast<__half*>(biases2);
  if (dtype == B2F_BF16)
    return requant_dispatch<TagBF16>(wq, rows, cols_u32, scales, biases, n_groups, int(wpg), packed, s2, b2, st);
  if (dtype == B2F_F16)
    return requant_dispatch<TagF16>(wq, rows, cols_u32, scales, biases, n_groups, int(wpg), packed, s2, b2, st);
  if (dtype == B2F_F32)
    return requant_dispatch<TagF32>(wq, rows, cols_u32, scales, biases, n_groups, int(wpg), packed, s2, b2, st);
  return B2F_ERR_UNSUPPORTED;
}

int b2f_dequant_2bit(const uint8_t* packed, int64_t packed_ld, const void* scales2, const void* biases2,
                     int64_t n_groups, int64_t rows, int64_t n_values_per_row, float* out, void* stream) {
  if (rows < 0 || n_values_per_row <= 0 || n_groups <= 0 || n_values_per_row % n_groups != 0)
    return B2F_ERR_INVALID;
  if (packed_ld * 4 < n_values_per_row) return B2F_ERR_INVALID;
  if (rows == 0) return B2F_OK;
  if (!packed || !scales2 || !biases2 || !out) return B2F_ERR_INVALID;
  const int64_t total = rows * n_values_per_row;
  dequant_2bit_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(
      packed, packed_ld, static_cast<const __half*>(scales2), static_cast<const __half*>(biases2), n_groups, rows,
      n_values_per_row, out);
  return check_launch();
}

int b2f_fake_quant_sym(const void* w, int dtype, int64_t n, int bits, float* out, float* absmax_out,
                       void* stream) {
  if (n < 0 || !(bits == 4 || bits == 8)) return bits == 4 || bits == 8 ? B2F_ERR_INVALID : B2F_ERR_UNSUPPORTED;
  if (!absmax_out || (n > 0 && (!w || !out))) return B2F_ERR_INVALID;
  if (!aligned(absmax_out, 4)) return B2F_ERR_ALIGN;
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(absmax_out, 0, sizeof(float), st) != cudaSuccess) return check_launch();
  if (n == 0) return B2F_OK;
  const float qmax = bits <= 4 ? 7.0f : 127.0f;
  const float qmin = bits <= 4 ? -8.0f : -128.0f;
  unsigned int* am = reinterpret_cast<unsigned int*>(absmax_out);
  const int grid = grid_for(n, 256);
  if (dtype == B2F_BF16) {
    auto p = static_cast<const __nv_bfloat16*>(w);
    absmax_kernel<TagBF16><<<grid, 256, 0, st>>>(p, n, am);
    fake_quant_kernel<TagBF16><<<grid, 256, 0, st>>>(p, n, am, qmin, qmax, out);
  } else if (dtype == B2F_F16) {
    auto p = static_cast<const __half*>(w);
    absmax_kernel<TagF16><<<grid, 256, 0, st>>>(p, n, am);
    fake_quant_kernel<TagF16><<<grid, 256, 0, st>>>(p, n, am, qmin, qmax, out);
  } else if (dtype == B2F_F32) {
    auto p = static_cast<const float*>(w);
    absmax_kernel<TagF32><<<grid, 256, 0, st>>>(p, n, am);
    fake_quant_kernel<TagF32><<<grid, 256, 0, st>>>(p, n, am, qmin, qmax, out);
  } else {
    return B2F_ERR_UNSUPPORTED;
  }
  return check_launch();
}

}  // extern "C"
