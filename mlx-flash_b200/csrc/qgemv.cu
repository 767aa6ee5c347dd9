// (b) dequant-fused GEMV for the MLX affine format, dense and grouped
// (routed experts), with the SwitchGLU gate/up pair fused.
//
// Memory-bound design (decode: M <= 16..32 tokens per weight tile):
//  * A CTA owns a run of 16-row blocks of one weight matrix (one expert) and
//    one tile of <= 8*NT tokens.  Its NW warps split K: warp w owns GW
//    consecutive quantization groups.  The tile's activations for those
//    groups are loaded ONCE into registers as bf16 MMA B-fragments and stay
//    there while the weight rows stream past ("activations stationary").
//  * Weights are read with 8/16-byte vector loads of packed words and
//    unpacked in registers straight into bf16 A-fragments with one lop3 per
//    two values: (0x4300 | q) is the bf16 number 128+q.  For 8-bit words the
//    high nibble goes through (0x4500 | hi) = 2048 + 16*hi, so both halves
//    accumulate into the same fp32 accumulator.
//  * Each MMA k-step stays inside one quantization group, so the group's
//    scale and bias are applied once per group to the fp32 partial:
//        y += s * sum_k x_k*(OFF + q_k) + (b - OFF*s) * sum_k x_k
//    (OFF = 128 for 4-bit, 2176 for 8-bit), i.e. exactly q*s+b with fp32
//    accumulation -- the same factorisation MLX's qmv uses.
//  * The per-warp partial tiles are reduced across warps through shared
//    memory in a fixed order (deterministic), then written as bf16.
#include "common.cuh"

namespace b2f {

struct GemvParams {
  const __nv_bfloat16* x;
  int64_t ldx;
  const int32_t* x_row_index;
  int64_t x_row_div;
  int64_t M;  // dense: number of x rows
  const uint32_t* w[2];
  const __nv_bfloat16* s[2];
  const __nv_bfloat16* b[2];
  int64_t w_estride;   // words per expert matrix
  int64_t sb_estride;  // scale elements per expert matrix
  int64_t N, K;
  const __nv_bfloat16* residual;
  __nv_bfloat16* out;
  int64_t ldo;
  const int32_t* slot_count;  // grouped mode (else nullptr)
  const int4* slots;
  const int32_t* sorted;
  int tile;
  int rb_per_chunk;
};

template <int BITS>
struct WordFrag;

// 4-bit: a word holds 8 consecutive k.  R_i = (e_i, e_{i+4}) as bf16 128+q.
template <>
struct WordFrag<4> {
  static __device__ __forceinline__ void unpack(uint32_t w, uint32_t (&R)[4]) {
    R[0] = and_or(w, 0x000F000Fu, 0x43004300u);
    R[1] = and_or(w >> 4, 0x000F000Fu, 0x43004300u);
    R[2] = and_or(w >> 8, 0x000F000Fu, 0x43004300u);
    R[3] = and_or(w >> 12, 0x000F000Fu, 0x43004300u);
  }
};

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + __expf(-g)) * u; }

template <int BITS, int GS, int NT, int GW, int MAT>
__global__ void __launch_bounds__(512, 1) qgemv_kernel(const GemvParams p) {
  constexpr int STEPS = GS / 16;           // MMA k-steps per group
  constexpr int CHUNK_K = GS / 4;          // k values per thread per group
  constexpr int CW = CHUNK_K * BITS / 32;  // packed words per thread per group per row
  constexpr int XV = CHUNK_K / 8;          // 16-byte activation loads per thread per group
  constexpr float OFF = BITS == 4 ? 128.f : 2176.f;
  constexpr int TILE_COLS = 8 * NT;

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int NW = blockDim.x >> 5;
  const int r = lane >> 2, c = lane & 3;
  const int G = int(p.K / GS);
  const int64_t words_per_row = p.K * BITS / 32;

  int expert = 0, tok_begin, n_tok;
  if (p.slots) {
    if (int(blockIdx.y) >= *p.slot_count) return;
    const int4 sl = p.slots[blockIdx.y];
    expert = sl.x;
    tok_begin = sl.y;
    n_tok = sl.z;
  } else {
    tok_begin = int(blockIdx.y) * p.tile;
    n_tok = int(min(int64_t(p.tile), p.M - tok_begin));
  }

  // ---- activation B-fragments and per-group activation sums -----------
  uint32_t bfr[GW][NT][STEPS][2];
  float xsum[GW][NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int ti = nt * 8 + r;
    const bool tvalid = ti < n_tok;
    int64_t xrow = 0;
    if (tvalid) {
      if (p.slots) {
        const int a = p.sorted[tok_begin + ti];
        xrow = p.x_row_index ? int64_t(p.x_row_index[a]) : int64_t(a) / p.x_row_div;
      } else {
        xrow = tok_begin + ti;
      }
    }
#pragma unroll
    for (int j = 0; j < GW; ++j) {
      const int g = warp * GW + j;
      const bool valid = tvalid && g < G;
      uint32_t xr[XV * 4];
      if (valid) {
        const uint4* src = reinterpret_cast<const uint4*>(p.x + xrow * p.ldx + int64_t(g) * GS + c * CHUNK_K);
#pragma unroll
        for (int v = 0; v < XV; ++v) {
          const uint4 q = src[v];
          xr[4 * v + 0] = q.x;
          xr[4 * v + 1] = q.y;
          xr[4 * v + 2] = q.z;
          xr[4 * v + 3] = q.w;
        }
      } else {
#pragma unroll
        for (int v = 0; v < XV * 4; ++v) xr[v] = 0u;
      }
      float part = 0.f;
#pragma unroll
      for (int v = 0; v < XV * 4; ++v) {
        const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&xr[v]);
        part += __low2float(h) + __high2float(h);
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      xsum[j][nt][0] = __shfl_sync(0xffffffffu, part, 8 * c);
      xsum[j][nt][1] = __shfl_sync(0xffffffffu, part, 8 * c + 4);
      if constexpr (BITS == 4) {
        // word wi covers 8 k: regs X01,X23,X45,X67 = xr[4wi .. 4wi+3]
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
          const int wi = s >> 1;
          const uint32_t* xw = &xr[4 * wi];
          if ((s & 1) == 0) {
            bfr[j][nt][s][0] = prmt(xw[0], xw[2], 0x5410u);  // (x0, x4)
            bfr[j][nt][s][1] = prmt(xw[0], xw[2], 0x7632u);  // (x1, x5)
          } else {
            bfr[j][nt][s][0] = prmt(xw[1], xw[3], 0x5410u);  // (x2, x6)
            bfr[j][nt][s][1] = prmt(xw[1], xw[3], 0x7632u);  // (x3, x7)
          }
        }
      } else {
        // word s covers 4 k: regs X01, X23 = xr[2s], xr[2s+1]
#pragma unroll
        for (int s = 0; s < STEPS; ++s) {
          bfr[j][nt][s][0] = prmt(xr[2 * s], xr[2 * s + 1], 0x5410u);  // (x0, x2)
          bfr[j][nt][s][1] = prmt(xr[2 * s], xr[2 * s + 1], 0x7632u);  // (x1, x3)
        }
      }
    }
  }

  // ---- stream the weight rows ------------------------------------------
  extern __shared__ float red[];  // [NW][MAT][16][TILE_COLS]
  const int64_t n_rb = (p.N + 15) / 16;
  const int64_t rb_begin = int64_t(blockIdx.x) * p.rb_per_chunk;
  const int64_t rb_end = min(rb_begin + p.rb_per_chunk, n_rb);

  // sv packs (scale, bias) of one row/group as a bf16x2 (scale in the low half)
  uint32_t wcur[MAT][GW][2][CW], wnext[MAT][GW][2][CW];
  uint32_t scur[MAT][GW][2], snext[MAT][GW][2];

  auto load_rb = [&](int64_t rb, uint32_t (&wv)[MAT][GW][2][CW], uint32_t (&sv)[MAT][GW][2]) {
#pragma unroll
    for (int m = 0; m < MAT; ++m) {
      const uint32_t* wbase = p.w[m] + int64_t(expert) * p.w_estride;
      const uint16_t* sbase = reinterpret_cast<const uint16_t*>(p.s[m]) + int64_t(expert) * p.sb_estride;
      const uint16_t* bbase = reinterpret_cast<const uint16_t*>(p.b[m]) + int64_t(expert) * p.sb_estride;
#pragma unroll
      for (int j = 0; j < GW; ++j) {
        const int g = warp * GW + j;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int64_t row = rb * 16 + r + 8 * h;
          if (g < G && row < p.N) {
            const uint32_t* src = wbase + row * words_per_row + int64_t(g) * (GS * BITS / 32) + c * CW;
            if constexpr (CW == 1) {
              wv[m][j][h][0] = src[0];
            } else if constexpr (CW == 2) {
              const uint2 q = *reinterpret_cast<const uint2*>(src);
              wv[m][j][h][0] = q.x;
              wv[m][j][h][1] = q.y;
            } else {
#pragma unroll
              for (int v = 0; v < CW / 4; ++v) {
                const uint4 q = reinterpret_cast<const uint4*>(src)[v];
                wv[m][j][h][4 * v + 0] = q.x;
                wv[m][j][h][4 * v + 1] = q.y;
                wv[m][j][h][4 * v + 2] = q.z;
                wv[m][j][h][4 * v + 3] = q.w;
              }
            }
            sv[m][j][h] = uint32_t(sbase[row * G + g]) | (uint32_t(bbase[row * G + g]) << 16);
          } else {
#pragma unroll
            for (int v = 0; v < CW; ++v) wv[m][j][h][v] = 0u;
            sv[m][j][h] = 0u;
          }
        }
      }
    }
  };

  if (rb_begin < rb_end) load_rb(rb_begin, wcur, scur);
  for (int64_t rb = rb_begin; rb < rb_end; ++rb) {
    if (rb + 1 < rb_end) load_rb(rb + 1, wnext, snext);

    float acc[MAT][NT][4];
#pragma unroll
    for (int m = 0; m < MAT; ++m)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[m][nt][i] = 0.f;

#pragma unroll
    for (int j = 0; j < GW; ++j) {
      if (warp * GW + j >= G) continue;
#pragma unroll
      for (int m = 0; m < MAT; ++m) {
        float ag[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) ag[nt][i] = 0.f;
        if constexpr (BITS == 4) {
#pragma unroll
          for (int wi = 0; wi < CW; ++wi) {
            uint32_t R0[4], R1[4];
            WordFrag<4>::unpack(wcur[m][j][0][wi], R0);
            WordFrag<4>::unpack(wcur[m][j][1][wi], R1);
#pragma unroll
            for (int hs = 0; hs < 2; ++hs) {
              const int s = 2 * wi + hs;
              const uint32_t a[4] = {R0[2 * hs], R1[2 * hs], R0[2 * hs + 1], R1[2 * hs + 1]};
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) mma_bf16_16816(ag[nt], a, bfr[j][nt][s]);
            }
          }
        } else {
#pragma unroll
          for (int s = 0; s < STEPS; ++s) {
            const uint32_t w0 = wcur[m][j][0][s], w1 = wcur[m][j][1][s];
            const uint32_t lo[4] = {and_or(w0, 0x000F000Fu, 0x43004300u), and_or(w1, 0x000F000Fu, 0x43004300u),
                                    and_or(w0 >> 8, 0x000F000Fu, 0x43004300u),
                                    and_or(w1 >> 8, 0x000F000Fu, 0x43004300u)};
            const uint32_t hi[4] = {and_or(w0 >> 4, 0x000F000Fu, 0x45004500u),
                                    and_or(w1 >> 4, 0x000F000Fu, 0x45004500u),
                                    and_or(w0 >> 12, 0x000F000Fu, 0x45004500u),
                                    and_or(w1 >> 12, 0x000F000Fu, 0x45004500u)};
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              mma_bf16_16816(ag[nt], lo, bfr[j][nt][s]);
              mma_bf16_16816(ag[nt], hi, bfr[j][nt][s]);
            }
          }
        }
        // group epilogue: y += s*acc + (b - OFF*s) * sum(x)
        const float s0 = __uint_as_float(scur[m][j][0] << 16);
        const float s1 = __uint_as_float(scur[m][j][1] << 16);
        const float c0 = __uint_as_float(scur[m][j][0] & 0xFFFF0000u) - OFF * s0;
        const float c1 = __uint_as_float(scur[m][j][1] & 0xFFFF0000u) - OFF * s1;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          acc[m][nt][0] += s0 * ag[nt][0] + c0 * xsum[j][nt][0];
          acc[m][nt][1] += s0 * ag[nt][1] + c0 * xsum[j][nt][1];
          acc[m][nt][2] += s1 * ag[nt][2] + c1 * xsum[j][nt][0];
          acc[m][nt][3] += s1 * ag[nt][3] + c1 * xsum[j][nt][1];
        }
      }
    }

    // ---- cross-warp reduction (fixed order) and store -----------------
#pragma unroll
    for (int m = 0; m < MAT; ++m)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = r + 8 * (i >> 1);
          const int col = nt * 8 + 2 * c + (i & 1);
          red[((warp * MAT + m) * 16 + row) * TILE_COLS + col] = acc[m][nt][i];
        }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 16 * TILE_COLS; idx += blockDim.x) {
      const int col = idx >> 4, row = idx & 15;
      const int64_t n = rb * 16 + row;
      if (col < n_tok && n < p.N) {
        float v0 = 0.f, v1 = 0.f;
        for (int w = 0; w < NW; ++w) {
          v0 += red[((w * MAT + 0) * 16 + row) * TILE_COLS + col];
          if constexpr (MAT == 2) v1 += red[((w * MAT + 1) * 16 + row) * TILE_COLS + col];
        }
        const int64_t orow = p.slots ? int64_t(p.sorted[tok_begin + col]) : int64_t(tok_begin + col);
        float v = (MAT == 2) ? silu_mul(v0, v1) : v0;
        if (p.residual) v += __bfloat162float(p.residual[orow * p.ldo + n]);
        p.out[orow * p.ldo + n] = __float2bfloat16_rn(v);
      }
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < MAT; ++m)
#pragma unroll
      for (int j = 0; j < GW; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int v = 0; v < CW; ++v) wcur[m][j][h][v] = wnext[m][j][h][v];
          scur[m][j][h] = snext[m][j][h];
        }
  }
}

// ---- MoE plan: counting sort of assignments by expert, cut into tiles ----
struct PlanLayout {
  int64_t off_hdr, off_counts, off_offsets, off_cursor, off_soff, off_sorted, off_slots, total;
};

static int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

static int64_t plan_max_slots(int64_t A, int64_t E, int tile) {
  const int64_t ne = A < E ? A : E;
  return ne + A / tile + 1;
}

static PlanLayout plan_layout(int64_t A, int64_t E, int tile) {
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
__device__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
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

__global__ void __launch_bounds__(1024) moe_plan_kernel(const int32_t* __restrict__ expert_of, int A, int E,
                                                        int tile, char* ws, PlanLayout L,
                                                        int32_t* status_out) {
  int32_t* hdr = reinterpret_cast<int32_t*>(ws + L.off_hdr);
  int32_t* counts = reinterpret_cast<int32_t*>(ws + L.off_counts);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.off_offsets);
  int32_t* cursor = reinterpret_cast<int32_t*>(ws + L.off_cursor);
  int32_t* soff = reinterpret_cast<int32_t*>(ws + L.off_soff);
  int32_t* sorted = reinterpret_cast<int32_t*>(ws + L.off_sorted);
  int4* slots = reinterpret_cast<int4*>(ws + L.off_slots);
  __shared__ int warp_tot[32];
  __shared__ int total;
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    counts[e] = 0;
    cursor[e] = 0;
  }
  __syncthreads();
  for (int a = threadIdx.x; a < A; a += blockDim.x) {
    const int e = expert_of[a];
    if (e < 0 || e >= E) {
      bad = 1;
    } else {
      atomicAdd(&counts[e], 1);
    }
  }
  __syncthreads();
  // exclusive scans over experts (chunks of blockDim.x)
  int run = 0, srun = 0;
  for (int base = 0; base < E; base += blockDim.x) {
    const int e = base + threadIdx.x;
    const int cnt = e < E ? counts[e] : 0;
    const int ns = (cnt + tile - 1) / tile;
    const int ex = block_exclusive_scan(cnt, warp_tot, &total);
    const int t1 = total;
    __syncthreads();
    const int sx = block_exclusive_scan(ns, warp_tot, &total);
    const int t2 = total;
    if (e < E) {
      offsets[e] = run + ex;
      soff[e] = srun + sx;
    }
    run += t1;
    srun += t2;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    offsets[E] = run;
    soff[E] = srun;
    hdr[0] = srun;
    hdr[1] = bad ? B2F_ERR_INVALID : B2F_OK;
    if (status_out) *status_out = hdr[1];
  }
  __syncthreads();
  for (int a = threadIdx.x; a < A; a += blockDim.x) {
    const int e = expert_of[a];
    if (e >= 0 && e < E) {
      const int pos = offsets[e] + atomicAdd(&cursor[e], 1);
      sorted[pos] = a;
    }
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int cnt = counts[e];
    for (int j = 0, s = soff[e]; j * tile < cnt; ++j, ++s)
      slots[s] = make_int4(e, offsets[e] + j * tile, min(tile, cnt - j * tile), 0);
  }
}

// ---- launcher ------------------------------------------------------------
template <int BITS, int GS, int NT, int GW, int MAT>
static int launch_gemv_cfg(const GemvParams& p, int64_t slots_grid, int NW, cudaStream_t st) {
  const int64_t n_rb = (p.N + 15) / 16;
  const int64_t chunks = (n_rb + p.rb_per_chunk - 1) / p.rb_per_chunk;
  if (chunks > 0x7fffffff || slots_grid > 65535) return B2F_ERR_UNSUPPORTED;
  const int smem = NW * MAT * 16 * 8 * NT * int(sizeof(float));
  const dim3 grid{unsigned(chunks), unsigned(slots_grid), 1u};
  auto kern = qgemv_kernel<BITS, GS, NT, GW, MAT>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return B2F_ERR_CUDA;
    }
  }
  kern<<<grid, NW * 32, smem, st>>>(p);
  return check_launch();
}

template <int BITS, int GS, int NT, int MAT>
static int launch_gemv_gw(const GemvParams& p, int64_t slots_grid, cudaStream_t st) {
  const int G = int(p.K / GS);
  if (G <= 16) return launch_gemv_cfg<BITS, GS, NT, 1, MAT>(p, slots_grid, G, st);
  if (G <= 32) return launch_gemv_cfg<BITS, GS, NT, 2, MAT>(p, slots_grid, (G + 1) / 2, st);
  if constexpr (NT == 1 && GS <= 64) {
    if (G <= 64) return launch_gemv_cfg<BITS, GS, NT, 4, MAT>(p, slots_grid, (G + 3) / 4, st);
  }
  return B2F_ERR_UNSUPPORTED;
}

template <int NT, int MAT>
static int launch_gemv_nt(const GemvParams& p, int bits, int gs, int64_t slots_grid, cudaStream_t st) {
  if (bits == 4) {
    if (gs == 32) return launch_gemv_gw<4, 32, NT, MAT>(p, slots_grid, st);
    if (gs == 64) return launch_gemv_gw<4, 64, NT, MAT>(p, slots_grid, st);
    if (gs == 128) return launch_gemv_gw<4, 128, NT, MAT>(p, slots_grid, st);
  } else if (bits == 8) {
    if (gs == 32) return launch_gemv_gw<8, 32, NT, MAT>(p, slots_grid, st);
    if (gs == 64) return launch_gemv_gw<8, 64, NT, MAT>(p, slots_grid, st);
    if (gs == 128) return launch_gemv_gw<8, 128, NT, MAT>(p, slots_grid, st);
  }
  return B2F_ERR_UNSUPPORTED;
}

static int launch_gemv(const GemvParams& p, int bits, int gs, int nt, int mat, int64_t slots_grid,
                       cudaStream_t st) {
  if (mat == 1) {
    if (nt == 1) return launch_gemv_nt<1, 1>(p, bits, gs, slots_grid, st);
    if (nt == 2) return launch_gemv_nt<2, 1>(p, bits, gs, slots_grid, st);
  } else {
    if (nt == 1) return launch_gemv_nt<1, 2>(p, bits, gs, slots_grid, st);
    if (nt == 2) return launch_gemv_nt<2, 2>(p, bits, gs, slots_grid, st);
  }
  return B2F_ERR_UNSUPPORTED;
}

// Row-blocks per CTA so that the grid has roughly `target` CTAs.
static int pick_rb_per_chunk(int64_t n_rb, int64_t slots, int64_t target) {
  int64_t want = (n_rb * slots + target - 1) / target;
  if (want < 1) want = 1;
  if (want > n_rb) want = n_rb;
  return int(want);
}

static int check_gemv_shape(int64_t N, int64_t K, int bits, int gs) {
  if (!(bits == 4 || bits == 8)) return B2F_ERR_UNSUPPORTED;
  if (!(gs == 32 || gs == 64 || gs == 128)) return B2F_ERR_UNSUPPORTED;
  if (N < 0 || K <= 0 || K % gs != 0) return B2F_ERR_INVALID;
  if (K / gs > 64) return B2F_ERR_UNSUPPORTED;
  return B2F_OK;
}

}  // namespace b2f

using namespace b2f;

extern "C" {

int b2f_qgemv_affine(const void* x, int64_t ldx, int64_t M, const uint32_t* wq, const void* scales,
                     const void* biases, int64_t N, int64_t K, int bits, int group_size,
                     const void* residual, void* y, int64_t ldy, void* stream) {
  int rc = check_gemv_shape(N, K, bits, group_size);
  if (rc != B2F_OK) return rc;
  if (M < 0) return B2F_ERR_INVALID;
  if (M == 0 || N == 0) return B2F_OK;
  if (!x || !wq || !scales || !biases || !y) return B2F_ERR_INVALID;
  if (ldx < K || ldy < N) return B2F_ERR_INVALID;
  if (!aligned(x, 16) || (ldx % 8) != 0 || !aligned(wq, 16)) return B2F_ERR_ALIGN;
  GemvParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.M = M;
  p.w[0] = wq;
  p.s[0] = static_cast<const __nv_bfloat16*>(scales);
  p.b[0] = static_cast<const __nv_bfloat16*>(biases);
  p.N = N;
  p.K = K;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.out = static_cast<__nv_bfloat16*>(y);
  p.ldo = ldy;
  // two 8-token MMA columns per CTA while the B fragments fit in registers
  const int nt = (M <= 8 || K / group_size > 32) ? 1 : 2;
  p.tile = 8 * nt;
  const int64_t slots = (M + p.tile - 1) / p.tile;
  const int64_t n_rb = (N + 15) / 16;
  p.rb_per_chunk = pick_rb_per_chunk(n_rb, slots, 148 * 2);
  return launch_gemv(p, bits, group_size, nt, 1, slots, as_stream(stream));
}

int64_t b2f_moe_plan_workspace_bytes(int64_t A, int64_t E, int tile) {
  if (A < 0 || E <= 0 || tile <= 0) return 0;
  return plan_layout(A, E, tile).total;
}

int64_t b2f_moe_plan_max_slots(int64_t A, int64_t E, int tile) {
  if (A < 0 || E <= 0 || tile <= 0) return 0;
  return plan_max_slots(A, E, tile);
}

int b2f_moe_plan(const int32_t* expert_of, int64_t A, int64_t E, int tile, void* workspace,
                 int64_t workspace_bytes, int32_t* status_out, void* stream) {
  if (A < 0 || E <= 0 || !(tile == 8 || tile == 16 || tile == 32)) return B2F_ERR_INVALID;
  if (A > 0x3fffffff || E > 65535) return B2F_ERR_UNSUPPORTED;
  PlanLayout L = plan_layout(A, E, tile);
  if (!workspace || workspace_bytes < L.total) return B2F_ERR_WORKSPACE;
  if (A > 0 && !expert_of) return B2F_ERR_INVALID;
  if (!aligned(workspace, 16)) return B2F_ERR_ALIGN;
  moe_plan_kernel<<<1, 1024, 0, as_stream(stream)>>>(expert_of, int(A), int(E), tile,
                                                     static_cast<char*>(workspace), L, status_out);
  return check_launch();
}

int b2f_gather_qgemv_affine(const void* x, int64_t ldx, const int32_t* x_row_index,
                            int64_t x_row_div, int64_t A, int64_t E, const uint32_t* w_gate,
                            const void* s_gate, const void* b_gate, const uint32_t* w_up,
                            const void* s_up, const void* b_up, int64_t N, int64_t K, int bits,
                            int group_size, int tile, const void* plan_workspace,
                            int64_t plan_workspace_bytes, void* out, int64_t ldo, void* stream) {
  int rc = check_gemv_shape(N, K, bits, group_size);
  if (rc != B2F_OK) return rc;
  if (A < 0 || E <= 0) return B2F_ERR_INVALID;
  if (A == 0 || N == 0) return B2F_OK;
  if (!(tile == 8 || tile == 16)) return B2F_ERR_UNSUPPORTED;
  if (tile == 16 && K / group_size > 32) return B2F_ERR_UNSUPPORTED;
  if (!x || !w_gate || !s_gate || !b_gate || !out) return B2F_ERR_INVALID;
  if (w_up && (!s_up || !b_up)) return B2F_ERR_INVALID;
  if (!x_row_index && x_row_div <= 0) return B2F_ERR_INVALID;
  if (ldx < K || ldo < N) return B2F_ERR_INVALID;
  if (!aligned(x, 16) || (ldx % 8) != 0 || !aligned(w_gate, 16) || (w_up && !aligned(w_up, 16)))
    return B2F_ERR_ALIGN;
  PlanLayout L = plan_layout(A, E, tile);
  if (!plan_workspace || plan_workspace_bytes < L.total) return B2F_ERR_WORKSPACE;
  const char* ws = static_cast<const char*>(plan_workspace);
  GemvParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.x_row_index = x_row_index;
  p.x_row_div = x_row_div > 0 ? x_row_div : 1;
  p.w[0] = w_gate;
  p.s[0] = static_cast<const __nv_bfloat16*>(s_gate);
  p.b[0] = static_cast<const __nv_bfloat16*>(b_gate);
  p.w[1] = w_up;
  p.s[1] = static_cast<const __nv_bfloat16*>(s_up);
  p.b[1] = static_cast<const __nv_bfloat16*>(b_up);
  p.w_estride = N * K * bits / 32;
  p.sb_estride = N * (K / group_size);
  p.N = N;
  p.K = K;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.slot_count = reinterpret_cast<const int32_t*>(ws + L.off_hdr);
  p.slots = reinterpret_cast<const int4*>(ws + L.off_slots);
  p.sorted = reinterpret_cast<const int32_t*>(ws + L.off_sorted);
  p.tile = tile;
  const int64_t max_slots = plan_max_slots(A, E, tile);
  const int64_t n_rb = (N + 15) / 16;
  const int64_t exp_slots = (A < E ? A : E);
  p.rb_per_chunk = pick_rb_per_chunk(n_rb, exp_slots, 148 * 3);
  return launch_gemv(p, bits, group_size, tile / 8, w_up ? 2 : 1, max_slots, as_stream(stream));
}

}  // extern "C"
