// (b) dequant-fused GEMV for the MLX affine format, dense and grouped
// (routed experts), with the SwitchGLU gate/up pair fused.
//
// Memory-bound design (decode: <= 16 tokens per weight pass):
//  * Work is the flattened sequence (token tile, 16-row block), split into
//    equal contiguous ranges, one per CTA (stream-K balance).
//  * A producer warp streams each 16-row block of packed words (plus its
//    scales/biases) into a STAGES-deep shared-memory ring with TMA bulk
//    copies (cp.async.bulk, completion on an mbarrier's transaction count)
//    and refills a stage once every consumer warp released it.
//  * Consumer warps split K by quantization group.  Each keeps the tile's
//    activations for its groups in registers as MMA B-fragments, reloaded
//    only when the token tile changes ("activations stationary").
//  * Packed words are unpacked in registers straight into bf16 A-fragments:
//    (0x4300 | q) is the bf16 number 128+q; the high nibble of an 8-bit code
//    goes through (0x4500 | hi) = 2048 + 16*hi.  Legacy warp MMAs
//    (mma.sync m16n8k16, fp32 accumulate) do the dot products.
//  * Each MMA k-step stays inside one quantization group, so scale and bias
//    are applied once per group to the fp32 partial:
//        y += s * sum_k x_k*(OFF + q_k) + (b - OFF*s) * sum_k x_k
//    (OFF = 128 for 4-bit, 2176 for 8-bit) -- exactly q*s+b with fp32
//    accumulation, the factorisation MLX's qmv uses.
//  * Per-warp partial tiles are reduced across warps through a padded,
//    double-buffered shared-memory tile in a fixed order (deterministic).
#include "common.cuh"
#include "plan.cuh"

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
  int32_t* err;  // optional: set to B2F_ERR_TIMEOUT if a bounded wait gave up
};

// Shared-memory plan of one launch (host-computed).
struct SmemPlan {
  int pitch;      // bytes per staged weight row (row_bytes padded against bank conflicts)
  int row_bytes;  // K*BITS/8
  int off_w[2], off_s[2], off_b[2];
  int stage_bytes, stages, red_off, red_buf_floats, flag_off, mbar_off;
};

constexpr int RED_PITCH = 20;  // floats per output column of a partial tile (16 rows; 20 = 4 mod 16)

// 4-bit: a word holds 8 consecutive k.  R_i = (e_i, e_{i+4}) as bf16 128+q.
__device__ __forceinline__ void unpack4(uint32_t w, uint32_t (&R)[4]) {
  R[0] = and_or(w, 0x000F000Fu, 0x43004300u);
  R[1] = and_or(w >> 4, 0x000F000Fu, 0x43004300u);
  R[2] = and_or(w >> 8, 0x000F000Fu, 0x43004300u);
  R[3] = and_or(w >> 12, 0x000F000Fu, 0x43004300u);
}

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + __expf(-g)) * u; }

template <int BITS, int GS, int NT, int GW, int MAT>
__global__ void __launch_bounds__(288, 1) qgemv_kernel(const GemvParams p, const SmemPlan L) {
  pdl_enter();
  constexpr int STEPS = GS / 16;           // MMA k-steps per group
  constexpr int CHUNK_K = GS / 4;          // k values per thread per group
  constexpr int CW = CHUNK_K * BITS / 32;  // packed words per thread per group per row
  constexpr int XV = CHUNK_K / 8;          // 16-byte activation loads per thread per group
  constexpr int GROUP_BYTES = GS * BITS / 8;
  constexpr float OFF = BITS == 4 ? 128.f : 2176.f;
  constexpr int TILE_COLS = 8 * NT;
  constexpr int OUTS = 16 * TILE_COLS;  // outputs per row block
  constexpr int MAX_OPT = 8;            // outputs per consumer thread (>= OUTS / 32)

  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int NW = int(blockDim.x >> 5) - 1;  // consumer warps; warp NW produces
  const int NC = NW * 32;
  const int r = lane >> 2, c = lane & 3;
  const int G = int(p.K / GS);
  const int64_t n_rb = (p.N + 15) / 16;
  const int n_slots = p.slots ? *p.slot_count : int((p.M + p.tile - 1) / p.tile);
  const int64_t W = int64_t(n_slots) * n_rb;
  const int64_t per = (W + gridDim.x - 1) / gridDim.x;
  const int64_t w_begin = int64_t(blockIdx.x) * per;
  const int64_t w_end = min(W, w_begin + per);
  if (w_begin >= w_end) return;
  const int n_iter = int(w_end - w_begin);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.mbar_off);
  uint64_t* empty = full + L.stages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.flag_off);
  float* red = reinterpret_cast<float*>(smem + L.red_off);

  auto slot_info = [&](int slot, int& expert, int& tok_begin, int& n_tok) {
    if (p.slots) {
      const int4 sl = p.slots[slot];
      expert = sl.x;
      tok_begin = sl.y;
      n_tok = sl.z;
    } else {
      expert = 0;
      tok_begin = slot * p.tile;
      n_tok = int(min(int64_t(p.tile), p.M - tok_begin));
    }
  };
  // scales/biases of a block go through TMA when the copy is 16-byte shaped
  auto sb_tma_ok = [&](int64_t e0, int rows) {
    return ((rows * G * 2) % 16) == 0 && aligned16(p.s[0] + e0) && aligned16(p.b[0] + e0) &&
           (MAT == 1 || (aligned16(p.s[1] + e0) && aligned16(p.b[1] + e0)));
  };

  if (tid == 0) {
    for (int s = 0; s < L.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();

  // =========================== producer warp ================================
  if (warp == NW) {
    if (lane == 0 && !producers_stalled()) {  // test control: stalled producers issue nothing
      for (int it = 0; it < n_iter; ++it) {
        const int s = it % L.stages;
        if (it >= L.stages) {
          if (*abort_flag || !mbar_wait_bounded(&empty[s], uint32_t(((it / L.stages) - 1) & 1))) {
            *abort_flag = 1;
            break;
          }
        }
        const int64_t widx = w_begin + it;
        const int slot = int(widx / n_rb);
        const int64_t rb = widx - int64_t(slot) * n_rb;
        int expert, tb, nt_;
        slot_info(slot, expert, tb, nt_);
        const int rows = int(min(int64_t(16), p.N - rb * 16));
        uint8_t* st = smem + s * L.stage_bytes;
        const int sbr = rows * G * 2;
        const int64_t e0 = int64_t(expert) * p.sb_estride + rb * 16 * G;
        const bool sb_tma = sb_tma_ok(e0, rows);
        const uint32_t bytes = uint32_t(MAT * rows * L.row_bytes + (sb_tma ? MAT * 2 * sbr : 0));
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&full[s], bytes);
#pragma unroll
        for (int m = 0; m < MAT; ++m) {
          const uint8_t* wb = reinterpret_cast<const uint8_t*>(p.w[m] + int64_t(expert) * p.w_estride) +
                              rb * 16 * int64_t(L.row_bytes);
          for (int rr = 0; rr < rows; ++rr)
            bulk_g2s(st + L.off_w[m] + rr * L.pitch, wb + int64_t(rr) * L.row_bytes, uint32_t(L.row_bytes),
                     &full[s]);
          if (sb_tma) {
            bulk_g2s(st + L.off_s[m], p.s[m] + e0, uint32_t(sbr), &full[s]);
            bulk_g2s(st + L.off_b[m], p.b[m] + e0, uint32_t(sbr), &full[s]);
          }
        }
      }
    }
    return;
  }

  // =========================== consumer warps ===============================
  uint32_t bfr[GW][NT][STEPS][2];
  float xsum[GW][NT][2];
  int64_t my_orow[MAX_OPT];
  int cur_slot = -1, expert = 0, tok_begin = 0, n_tok = 0;
  bool timed_out = false;

  for (int it = 0; it < n_iter; ++it) {
    const int64_t widx = w_begin + it;
    const int slot = int(widx / n_rb);
    const int64_t rb = widx - int64_t(slot) * n_rb;
    if (slot != cur_slot) {
      // (re)load this token tile's activations as register B-fragments
      cur_slot = slot;
      slot_info(slot, expert, tok_begin, n_tok);
#pragma unroll
      for (int k = 0; k < MAX_OPT; ++k) {
        const int idx = tid + k * NC;
        const int col = idx >> 4;
        my_orow[k] = -1;
        if (idx < OUTS && col < n_tok)
          my_orow[k] = p.slots ? int64_t(p.sorted[tok_begin + col]) : int64_t(tok_begin + col);
      }
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
            const uint4* src =
                reinterpret_cast<const uint4*>(p.x + xrow * p.ldx + int64_t(g) * GS + c * CHUNK_K);
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
#pragma unroll
            for (int s = 0; s < STEPS; ++s) {
              const uint32_t* xw = &xr[4 * (s >> 1)];
              if ((s & 1) == 0) {
                bfr[j][nt][s][0] = prmt(xw[0], xw[2], 0x5410u);  // (x0, x4)
                bfr[j][nt][s][1] = prmt(xw[0], xw[2], 0x7632u);  // (x1, x5)
              } else {
                bfr[j][nt][s][0] = prmt(xw[1], xw[3], 0x5410u);  // (x2, x6)
                bfr[j][nt][s][1] = prmt(xw[1], xw[3], 0x7632u);  // (x3, x7)
              }
            }
          } else {
#pragma unroll
            for (int s = 0; s < STEPS; ++s) {
              bfr[j][nt][s][0] = prmt(xr[2 * s], xr[2 * s + 1], 0x5410u);  // (x0, x2)
              bfr[j][nt][s][1] = prmt(xr[2 * s], xr[2 * s + 1], 0x7632u);  // (x1, x3)
            }
          }
        }
      }
    }

    // residual of this block's outputs, fetched before the math
    float resid[MAX_OPT];
#pragma unroll
    for (int k = 0; k < MAX_OPT; ++k) {
      resid[k] = 0.f;
      const int64_t n = rb * 16 + ((tid + k * NC) & 15);
      if (p.residual && my_orow[k] >= 0 && n < p.N)
        resid[k] = __bfloat162float(p.residual[my_orow[k] * p.ldo + n]);
    }

    const int s_idx = it % L.stages;
    if (!timed_out) {
      if (*abort_flag || !mbar_wait_bounded(&full[s_idx], uint32_t((it / L.stages) & 1))) {
        timed_out = true;
        *abort_flag = 1;
      }
    }
    const uint8_t* st = smem + s_idx * L.stage_bytes;
    const int rows = int(min(int64_t(16), p.N - rb * 16));
    const int64_t sb0 = int64_t(expert) * p.sb_estride + rb * 16 * G;
    const bool sb_tma = sb_tma_ok(sb0, rows);

    float acc[MAT][NT][4];
#pragma unroll
    for (int m = 0; m < MAT; ++m)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[m][nt][i] = 0.f;

#pragma unroll
    for (int j = 0; j < GW; ++j) {
      const int g = warp * GW + j;
      if (g >= G) continue;
#pragma unroll
      for (int m = 0; m < MAT; ++m) {
        uint32_t wv[2][CW];
        float sc[2], bi[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = r + 8 * h;
          const uint8_t* src = st + L.off_w[m] + row * L.pitch + g * GROUP_BYTES + c * CW * 4;
          if constexpr (CW == 1) {
            wv[h][0] = *reinterpret_cast<const uint32_t*>(src);
          } else if constexpr (CW == 2) {
            const uint2 q = *reinterpret_cast<const uint2*>(src);
            wv[h][0] = q.x;
            wv[h][1] = q.y;
          } else {
#pragma unroll
            for (int v = 0; v < CW / 4; ++v) {
              const uint4 q = reinterpret_cast<const uint4*>(src)[v];
              wv[h][4 * v + 0] = q.x;
              wv[h][4 * v + 1] = q.y;
              wv[h][4 * v + 2] = q.z;
              wv[h][4 * v + 3] = q.w;
            }
          }
          if (sb_tma) {
            sc[h] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(st + L.off_s[m])[row * G + g]);
            bi[h] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(st + L.off_b[m])[row * G + g]);
          } else if (row < rows) {
            const int64_t e0 = sb0 + int64_t(row) * G + g;
            sc[h] = __bfloat162float(p.s[m][e0]);
            bi[h] = __bfloat162float(p.b[m][e0]);
          } else {
            sc[h] = 0.f;
            bi[h] = 0.f;
          }
        }
        float ag[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) ag[nt][i] = 0.f;
        if constexpr (BITS == 4) {
#pragma unroll
          for (int wi = 0; wi < CW; ++wi) {
            uint32_t R0[4], R1[4];
            unpack4(wv[0][wi], R0);
            unpack4(wv[1][wi], R1);
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
            const uint32_t w0 = wv[0][s], w1 = wv[1][s];
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
        const float c0 = bi[0] - OFF * sc[0];
        const float c1 = bi[1] - OFF * sc[1];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          acc[m][nt][0] += sc[0] * ag[nt][0] + c0 * xsum[j][nt][0];
          acc[m][nt][1] += sc[0] * ag[nt][1] + c0 * xsum[j][nt][1];
          acc[m][nt][2] += sc[1] * ag[nt][2] + c1 * xsum[j][nt][0];
          acc[m][nt][3] += sc[1] * ag[nt][3] + c1 * xsum[j][nt][1];
        }
      }
    }
    // this warp is done reading stage s_idx
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s_idx]);

    // ---- cross-warp reduction (fixed order), double-buffered partials ------
    float* rbuf = red + (it & 1) * L.red_buf_floats;
#pragma unroll
    for (int m = 0; m < MAT; ++m)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = r + 8 * (i >> 1);
          const int col = nt * 8 + 2 * c + (i & 1);
          rbuf[((warp * MAT + m) * TILE_COLS + col) * RED_PITCH + row] = acc[m][nt][i];
        }
    named_sync(NC);
#pragma unroll
    for (int k = 0; k < MAX_OPT; ++k) {
      const int idx = tid + k * NC;
      if (idx >= OUTS) break;
      const int col = idx >> 4, row = idx & 15;
      const int64_t n = rb * 16 + row;
      if (my_orow[k] >= 0 && n < p.N) {
        float v0 = 0.f, v1 = 0.f;
        for (int w = 0; w < NW; ++w) {
          v0 += rbuf[((w * MAT + 0) * TILE_COLS + col) * RED_PITCH + row];
          if constexpr (MAT == 2) v1 += rbuf[((w * MAT + 1) * TILE_COLS + col) * RED_PITCH + row];
        }
        float v = (MAT == 2) ? silu_mul(v0, v1) : v0;
        v += resid[k];
        p.out[my_orow[k] * p.ldo + n] = __float2bfloat16_rn(v);
      }
    }
  }
  if (timed_out && lane == 0) report_timeout(p.err);
}

int64_t plan_slots_offset(int64_t A, int64_t E, int tile) { return plan_layout(A, E, tile).off_slots; }
int64_t plan_sorted_offset(int64_t A, int64_t E, int tile) { return plan_layout(A, E, tile).off_sorted; }

// ---- launcher ------------------------------------------------------------
static int g_num_sms = 0;

static int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
      g_num_sms = n;
    else
      g_num_sms = 148;
  }
  return g_num_sms;
}

template <int BITS, int GS, int NT, int GW, int MAT>
static int launch_gemv_cfg(const GemvParams& p, int64_t max_work, int NW, cudaStream_t st) {
  constexpr int CW = (GS / 4) * BITS / 32;
  SmemPlan L{};
  L.row_bytes = int(p.K * BITS / 8);
  // consecutive staged rows start 8 (32-bit loads: 4) or 16 banks apart
  const int extra = CW * 16 < 64 ? CW * 16 : 64;
  L.pitch = int(align_up(L.row_bytes, 128)) + extra;
  const int G = int(p.K / GS);
  const int sb = int(align_up(16 * G * 2, 16));
  int o = 0;
  for (int m = 0; m < MAT; ++m) {
    L.off_w[m] = o;
    o += 16 * L.pitch;
    L.off_s[m] = o;
    o += sb;
    L.off_b[m] = o;
    o += sb;
  }
  L.stage_bytes = int(align_up(o, 128));
  L.red_buf_floats = NW * MAT * 8 * NT * RED_PITCH;
  const int red_bytes = 2 * L.red_buf_floats * int(sizeof(float));
  const int budget = 220 * 1024;
  int stages = (budget - red_bytes - 512) / L.stage_bytes;
  if (stages > 8) stages = 8;
  if (stages < 2) return B2F_ERR_UNSUPPORTED;
  L.stages = stages;
  L.red_off = stages * L.stage_bytes;
  L.flag_off = int(align_up(L.red_off + red_bytes, 16));
  L.mbar_off = L.flag_off + 16;
  const int smem = L.mbar_off + 16 * stages;
  auto kern = qgemv_kernel<BITS, GS, NT, GW, MAT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return B2F_ERR_CUDA;
  }
  const int threads = (NW + 1) * 32;  // + one producer warp
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  int64_t grid = int64_t(num_sms()) * per_sm;
  if (grid > max_work) grid = max_work;
  if (grid < 1) grid = 1;
  return launch_kernel(kern, dim3{unsigned(grid)}, dim3{unsigned(threads)}, size_t(smem), st, p, L);
}

// Groups per warp: the smallest GW that keeps <= 8 consumer warps while the
// activation fragments (GW*NT*GS/8 registers) stay <= 64 registers.
template <int BITS, int GS, int NT, int MAT>
static int launch_gemv_gw(const GemvParams& p, int64_t max_work, cudaStream_t st) {
  const int G = int(p.K / GS);
  constexpr int MAXGW = (8 * 64 / GS) / NT;  // GW*NT*GS/8 <= 64
  if (G <= 8) return launch_gemv_cfg<BITS, GS, NT, 1, MAT>(p, max_work, G, st);
  if constexpr (MAXGW >= 2) {
    if (G <= 16) return launch_gemv_cfg<BITS, GS, NT, 2, MAT>(p, max_work, (G + 1) / 2, st);
  }
  if constexpr (MAXGW >= 4) {
    if (G <= 32) return launch_gemv_cfg<BITS, GS, NT, 4, MAT>(p, max_work, (G + 3) / 4, st);
  }
  if constexpr (MAXGW >= 8) {
    if (G <= 64) return launch_gemv_cfg<BITS, GS, NT, 8, MAT>(p, max_work, (G + 7) / 8, st);
  }
  // otherwise more warps with fewer groups each (<= 8 consumer warps still)
  return B2F_ERR_UNSUPPORTED;
}

template <int NT, int MAT>
static int launch_gemv_nt(const GemvParams& p, int bits, int gs, int64_t max_work, cudaStream_t st) {
  if (bits == 4) {
    if (gs == 32) return launch_gemv_gw<4, 32, NT, MAT>(p, max_work, st);
    if (gs == 64) return launch_gemv_gw<4, 64, NT, MAT>(p, max_work, st);
    if (gs == 128) return launch_gemv_gw<4, 128, NT, MAT>(p, max_work, st);
  } else if (bits == 8) {
    if (gs == 32) return launch_gemv_gw<8, 32, NT, MAT>(p, max_work, st);
    if (gs == 64) return launch_gemv_gw<8, 64, NT, MAT>(p, max_work, st);
    if (gs == 128) return launch_gemv_gw<8, 128, NT, MAT>(p, max_work, st);
  }
  return B2F_ERR_UNSUPPORTED;
}

// max_work: an upper bound on (token tiles x row blocks), used to cap the grid.
static int launch_gemv(const GemvParams& p, int bits, int gs, int nt, int mat, int64_t max_work,
                       cudaStream_t st) {
  if (mat == 1) {
    if (nt == 1) return launch_gemv_nt<1, 1>(p, bits, gs, max_work, st);
    if (nt == 2) return launch_gemv_nt<2, 1>(p, bits, gs, max_work, st);
  } else {
    if (nt == 1) return launch_gemv_nt<1, 2>(p, bits, gs, max_work, st);
    if (nt == 2) return launch_gemv_nt<2, 2>(p, bits, gs, max_work, st);
  }
  return B2F_ERR_UNSUPPORTED;
}

static int check_gemv_shape(int64_t N, int64_t K, int bits, int gs) {
  if (!(bits == 4 || bits == 8)) return B2F_ERR_UNSUPPORTED;
  if (!(gs == 32 || gs == 64 || gs == 128)) return B2F_ERR_UNSUPPORTED;
  if (N < 0 || K <= 0 || K % gs != 0) return B2F_ERR_INVALID;
  if (K / gs > 64) return B2F_ERR_UNSUPPORTED;
  return B2F_OK;
}

B2F_DEFINE_WAIT_CONTROLS(gemv)

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
  return launch_gemv(p, bits, group_size, nt, 1, slots * n_rb, as_stream(stream));
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
  if (A < 0 || E <= 0 || tile < 8 || tile > 256 || tile % 8 != 0) return B2F_ERR_INVALID;
  if (A > 0x3fffffff || E > 65535) return B2F_ERR_UNSUPPORTED;
  PlanLayout L = plan_layout(A, E, tile);
  if (!workspace || workspace_bytes < L.total) return B2F_ERR_WORKSPACE;
  if (A > 0 && !expert_of) return B2F_ERR_INVALID;
  if (!aligned(workspace, 16)) return B2F_ERR_ALIGN;
  return launch_kernel(moe_plan_kernel<DenseExperts>, dim3{1}, dim3{1024}, 0, as_stream(stream),
                       DenseExperts{expert_of}, int(A), int(E), tile, static_cast<char*>(workspace), L, status_out);
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
  // a bounded wait that gives up records B2F_ERR_TIMEOUT in the plan header's status word
  p.err = const_cast<int32_t*>(reinterpret_cast<const int32_t*>(ws + L.off_hdr)) + 1;
  p.slots = reinterpret_cast<const int4*>(ws + L.off_slots);
  p.sorted = reinterpret_cast<const int32_t*>(ws + L.off_sorted);
  p.tile = tile;
  const int64_t max_slots = plan_max_slots(A, E, tile);
  const int64_t n_rb = (N + 15) / 16;
  return launch_gemv(p, bits, group_size, tile / 8, w_up ? 2 : 1, max_slots * n_rb, as_stream(stream));
}

}  // extern "C"
