// (c) grouped expert GEMM on the 5th-generation tensor cores (tcgen05/TMEM):
// out[tokens, N] = x[tokens, K] . dequant(W[expert])^T for every (expert,
// token tile) slot of a MoE plan, optionally the SwitchGLU pair
// silu(x.Wg^T) * (x.Wu^T).  Used for prefill and for decode tiles with many
// tokens; the register-fragment GEMV (qgemv.cu) serves the small tiles.
//
// CTA = 128 weight rows (MMA M) x one token tile (MMA N = tokens rounded up to
// 16, <= TILE_N) x all of K, in K-chunks of 64 (one quantization group):
//   warp 0     TMA producer: 2-D tensor-map loads of the packed words of the
//              128 rows for the chunk (32B/64B-swizzled) into a ring.
//   warps 1-4  converters: dequantize row t of the chunk, w = q*s + b as one
//              bf16 rounding, into a 128B-swizzled K-major A tile (scales and
//              biases fetched one chunk ahead); afterwards the epilogue
//              (TMEM -> registers -> bf16 stores).
//   warps 6-7  x loaders (alternate chunks): gather the tile's token rows of x
//              for a chunk into the B tile (same K permutation), ahead of the math.
//   warp 5     MMA issuer (one thread): tcgen05.mma kind::f16, bf16 x bf16 ->
//              fp32 in TMEM, 4 x K16 per chunk per matrix; tcgen05.commit
//              frees the A/B stage and finally signals the accumulators.
// Within every 8-wide K slice both operands use the order (0,4,1,5,2,6,3,7),
// which is how the in-register nibble unpack produces pairs; the contraction
// over K is unchanged by a common permutation.
// Every mbarrier wait is bounded; on a timeout the kernel records
// B2F_ERR_TIMEOUT, skips the remaining work, and still frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tc_common.cuh"

namespace b2f {

struct TcParams {
  const __nv_bfloat16* x;
  int64_t ldx;
  const int32_t* x_row_index;
  int64_t x_row_div;
  int64_t M;  // dense mode: x rows
  const __nv_bfloat16* s[2];
  const __nv_bfloat16* b[2];
  int64_t sb_estride;  // scale elements per expert matrix
  int64_t N, K;        // N = weight rows per expert
  const __nv_bfloat16* residual;
  __nv_bfloat16* out;
  int64_t ldo;
  const int32_t* slot_count;  // grouped mode (else nullptr)
  const int4* slots;
  const int32_t* sorted;
  int tile;  // tokens per slot (<= TILE_N)
  int32_t* err;
  int pk_stages, ab_stages;
  int ksplit;      // dense mode: K is cut into ksplit ranges (grid z)
  float* partial;  // ksplit > 1: fp32 partials [ksplit][M][N]
};

template <int BITS, int MAT, int TILE_N>
__global__ void __launch_bounds__(256, 2) qgemm_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap tm0,
                                                         const __grid_constant__ CUtensorMap tm1) {
  pdl_enter();
  constexpr int PKB = TC_KC * BITS / 8;         // packed bytes per row per chunk (32 or 64)
  constexpr int PK_TILE = TC_M * PKB;           // per matrix
  constexpr int A_TILE = TC_M * TC_KC * 2;      // 16 KB per matrix
  constexpr int B_TILE = TILE_N * TC_KC * 2;    // TILE_N rows of 128 B
  constexpr uint32_t TMEM_COLS = (MAT * TILE_N <= 32) ? 32 : (MAT * TILE_N <= 64) ? 64 : (MAT * TILE_N <= 128) ? 128
                                 : (MAT * TILE_N <= 256) ? 256 : 512;
  constexpr int PK_SW_MASK = PKB / 16 - 1;      // 32B swizzle: 1 ; 64B swizzle: 3

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int PS = p.pk_stages, AS = p.ab_stages;

  // ---- slot of this CTA --------------------------------------------------
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
    if (n_tok <= 0) return;
  }
  const int n_pad = (n_tok + 15) & ~15;
  const int64_t m0 = int64_t(blockIdx.x) * TC_M;
  // this CTA's K range (split-K in dense mode): chunks [c_base, c_base + n_chunks)
  const int all_chunks = int(p.K / TC_KC);
  const int cps = (all_chunks + p.ksplit - 1) / p.ksplit;
  const int c_base = int(blockIdx.z) * cps;
  const int n_chunks = min(cps, all_chunks - c_base);
  if (n_chunks <= 0) return;

  // ---- shared memory carve-up (all tiles 1024-B aligned) ---------------------
  uint8_t* pk = smem;                                  // [PS][MAT][PK_TILE]
  uint8_t* ab = pk + PS * MAT * PK_TILE;               // [AS][MAT*A_TILE + B_TILE]
  const int ab_stride = MAT * A_TILE + B_TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ab + AS * ab_stride);
  uint64_t* pk_full = bars;
  uint64_t* pk_empty = pk_full + PS;
  uint64_t* ab_full = pk_empty + PS;
  uint64_t* ab_empty = ab_full + AS;
  uint64_t* acc_full = ab_empty + AS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int64_t* orow = reinterpret_cast<int64_t*>(tmem_slot + 4);  // [TILE_N]
  int64_t* xrow = orow + TILE_N;                               // [TILE_N]

  if (tid == 0) {
    for (int s = 0; s < PS; ++s) {
      mbar_init(&pk_full[s], 1);
      mbar_init(&pk_empty[s], 4);
    }
    for (int s = 0; s < AS; ++s) {
      mbar_init(&ab_full[s], 5);  // 4 converter warps + the x loader warp of that chunk
      mbar_init(&ab_empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  for (int n = tid; n < TILE_N; n += blockDim.x) {
    int64_t o = -1, xr = 0;
    if (n < n_tok) {
      if (p.slots) {
        const int a = p.sorted[tok_begin + n];
        o = a;
        xr = p.x_row_index ? int64_t(p.x_row_index[a]) : int64_t(a) / p.x_row_div;
      } else {
        o = tok_begin + n;
        xr = tok_begin + n;
      }
    }
    orow[n] = o;
    xrow[n] = xr;
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // =========================== TMA producer ================================
    if (lane == 0 && !producers_stalled()) {
      const int row0 = int(int64_t(expert) * p.N + m0);
      for (int c = 0; c < n_chunks; ++c) {
        const int s = c % PS;
        if (c >= PS && (*abort_flag || !mbar_wait_bounded(&pk_empty[s], uint32_t(((c / PS) - 1) & 1)))) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        mbar_arrive_expect_tx(&pk_full[s], uint32_t(MAT * PK_TILE));
        tma_load_2d(pk + (s * MAT + 0) * PK_TILE, &tm0, (c_base + c) * (PKB / 4), row0, &pk_full[s]);
        if constexpr (MAT == 2)
          tma_load_2d(pk + (s * MAT + 1) * PK_TILE, &tm1, (c_base + c) * (PKB / 4), row0, &pk_full[s]);
      }
    }
  } else if (warp == 5) {
    // =========================== MMA issuer ==================================
    if (lane == 0) {
      // kind::f16: D f32 (bit 4), A bf16 (bits 7-9 = 1), B bf16 (bits 10-12 = 1),
      // K-major A and B, N >> 3 at bit 17, M >> 4 at bit 24
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n_pad >> 3) << 17) |
                             (uint32_t(TC_M >> 4) << 24);
      for (int c = 0; c < n_chunks; ++c) {
        const int s = c % AS;
        if (*abort_flag || !mbar_wait_bounded(&ab_full[s], uint32_t((c / AS) & 1))) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        uint8_t* st = ab + s * ab_stride;
        const uint64_t bdesc = sw128_desc(st + MAT * A_TILE);
#pragma unroll
        for (int m = 0; m < MAT; ++m) {
          const uint64_t adesc = sw128_desc(st + m * A_TILE);
#pragma unroll
          for (int ks = 0; ks < TC_KC / 16; ++ks)  // +32 bytes per K16 step
            tc_mma(tmem + uint32_t(m * TILE_N), adesc + 2 * ks, bdesc + 2 * ks, idesc, (c > 0 || ks > 0) ? 1u : 0u);
        }
        tc_commit(&ab_empty[s]);
      }
      tc_commit(acc_full);
    }
  } else if (warp >= 6) {
    // =========================== x loaders (warps 6, 7: alternate chunks) =====
    // B tile: token rows of x for a chunk, K order (0,4,1,5,2,6,3,7) per 8.
    for (int c = warp - 6; c < n_chunks; c += 2) {
      const int s2 = c % AS;
      if (*abort_flag) break;
      if (c >= AS && !mbar_wait_bounded(&ab_empty[s2], uint32_t(((c / AS) - 1) & 1))) {
        *abort_flag = 1;
        break;
      }
      uint8_t* brow = ab + s2 * ab_stride + MAT * A_TILE;
      // batches of 8 16-byte vectors per lane: loads first, then permuted stores
      for (int base = 0; base < n_pad * 8; base += 256) {
        uint4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int idx = base + lane + 32 * i;
          const int n = idx >> 3, j = idx & 7;
          v[i] = make_uint4(0u, 0u, 0u, 0u);
          if (n < n_tok)
            v[i] = *reinterpret_cast<const uint4*>(p.x + xrow[n] * p.ldx + int64_t(c_base + c) * TC_KC + 8 * j);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int idx = base + lane + 32 * i;
          const int n = idx >> 3, j = idx & 7;
          if (n < n_pad) {
            const uint4 xv = v[i];
            *reinterpret_cast<uint4*>(brow + sw128_off(n, j)) =
                make_uint4(prmt(xv.x, xv.z, 0x5410u), prmt(xv.x, xv.z, 0x7632u), prmt(xv.y, xv.w, 0x5410u),
                           prmt(xv.y, xv.w, 0x7632u));
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ab_full[s2]);
    }
  } else {
    // =========================== converters (warps 1-4) ========================
    const int t = tid - 32;  // weight row within the tile (0..127)
    const int64_t grow = m0 + t;
    const bool row_ok = grow < p.N;
    const int64_t sb_row = int64_t(expert) * p.sb_estride + grow * (p.K / 64) + c_base;
    // scales/biases fetched two chunks ahead (raw bf16 bits)
    uint16_t sq[3][MAT], bq[3][MAT];
    const uint16_t* sp[MAT];
    const uint16_t* bp[MAT];
#pragma unroll
    for (int m = 0; m < MAT; ++m) {
      sp[m] = reinterpret_cast<const uint16_t*>(p.s[m]) + sb_row;
      bp[m] = reinterpret_cast<const uint16_t*>(p.b[m]) + sb_row;
#pragma unroll
      for (int d = 0; d < 2; ++d) {
        sq[d][m] = (row_ok && d < n_chunks) ? sp[m][d] : uint16_t(0);
        bq[d][m] = (row_ok && d < n_chunks) ? bp[m][d] : uint16_t(0);
      }
    }
    for (int c = 0; c < n_chunks; ++c) {
      float csc[MAT], cbi[MAT];
#pragma unroll
      for (int m = 0; m < MAT; ++m) {
        csc[m] = __uint_as_float(uint32_t(sq[0][m]) << 16);
        cbi[m] = __uint_as_float(uint32_t(bq[0][m]) << 16);
        sq[0][m] = sq[1][m];
        bq[0][m] = bq[1][m];
        sq[1][m] = (row_ok && c + 2 < n_chunks) ? sp[m][c + 2] : uint16_t(0);
        bq[1][m] = (row_ok && c + 2 < n_chunks) ? bp[m][c + 2] : uint16_t(0);
      }
      const int s1 = c % PS, s2 = c % AS;
      if (*abort_flag) break;
      if (!mbar_wait_bounded(&pk_full[s1], uint32_t((c / PS) & 1)) ||
          (c >= AS && !mbar_wait_bounded(&ab_empty[s2], uint32_t(((c / AS) - 1) & 1)))) {
        *abort_flag = 1;
        break;
      }
      uint8_t* st = ab + s2 * ab_stride;
#pragma unroll
      for (int m = 0; m < MAT; ++m) {
        const float sc = csc[m], bi = cbi[m];
        const uint32_t s2v = pack_bf16x2(sc, sc), b2v = pack_bf16x2(bi, bi);
        const uint8_t* prow = pk + (s1 * MAT + m) * PK_TILE + t * PKB;
        const int sw = (t * PKB >> 7) & PK_SW_MASK;  // TMA swizzle of this row
        uint8_t* arow = st + m * A_TILE;
        if constexpr (BITS == 4) {
          // 2 x 16 B = 8 words; word i -> A chunk i (k 8i..8i+7)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint4 q = *reinterpret_cast<const uint4*>(prow + ((h ^ sw) << 4));
            const uint32_t wds[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t w = wds[i];
              uint32_t o[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t qv = hsub2_bf(and_or(w >> (4 * j), 0x000F000Fu, 0x43004300u), 0x43004300u);
                o[j] = hfma2_bf(qv, s2v, b2v);  // (k j, k j+4)
              }
              *reinterpret_cast<uint4*>(arow + sw128_off(t, 4 * h + i)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
        } else {
          // 4 x 16 B = 16 words; words (2i, 2i+1) -> A chunk i; a word holds 4 k
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const uint4 q = *reinterpret_cast<const uint4*>(prow + ((h ^ sw) << 4));
            const uint32_t wds[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int ii = 0; ii < 2; ++ii) {
              const uint32_t wa = wds[2 * ii], wb = wds[2 * ii + 1];  // k 0..3, 4..7 of chunk
              uint32_t o[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                // (k j, k j+4): byte j of wa and byte j of wb
                const float qa = float((wa >> (8 * j)) & 0xFFu), qb = float((wb >> (8 * j)) & 0xFFu);
                o[j] = hfma2_bf(pack_bf16x2(qa, qb), s2v, b2v);
              }
              *reinterpret_cast<uint4*>(arow + sw128_off(t, 2 * h + ii)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
        }
      }
      fence_proxy_async_smem();  // generic-proxy stores -> tensor-core reads
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&ab_full[s2]);
        mbar_arrive(&pk_empty[s1]);
      }
    }

    // ---- epilogue: TMEM -> registers -> bf16 -------------------------------
    if (!*abort_flag && !mbar_wait_bounded(acc_full, 0u)) *abort_flag = 1;
    tc_fence_after();
    if (!*abort_flag) {
      const int q = warp & 3;  // TMEM lane quarter this warp may access
      const int row = 32 * q + lane;
      const int64_t gr = m0 + row;
      for (int n0 = 0; n0 < n_pad; n0 += 16) {
        uint32_t g[16], u[16];
        tmem_ld16(tmem + (uint32_t(32 * q) << 16) + uint32_t(n0), g);
        if constexpr (MAT == 2) tmem_ld16(tmem + (uint32_t(32 * q) << 16) + uint32_t(TILE_N + n0), u);
        if (gr < p.N) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = n0 + i;
            if (n < n_tok) {
              float v = __uint_as_float(g[i]);
              if constexpr (MAT == 2) v = silu_mul_tc(v, __uint_as_float(u[i]));
              const int64_t o = orow[n];
              if (p.partial) {
                p.partial[(int64_t(blockIdx.z) * p.M + o) * p.N + gr] = v;
              } else {
                if (p.residual) v += __bfloat162float(p.residual[o * p.ldo + gr]);
                p.out[o * p.ldo + gr] = __float2bfloat16_rn(v);
              }
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
  if (tid == 0 && *abort_flag) report_timeout(p.err);
}

// split-K: out[m, n] = bf16(sum_k partial[k, m, n] + residual[m, n])
__global__ void __launch_bounds__(256) splitk_finalize_kernel(const float* __restrict__ partial, int ksplit, int64_t M,
                                                              int64_t N, const __nv_bfloat16* __restrict__ residual,
                                                              __nv_bfloat16* __restrict__ out, int64_t ldo) {
  pdl_enter();
  const int64_t total = M * N;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    float v = 0.f;
    for (int k = 0; k < ksplit; ++k) v += partial[int64_t(k) * total + i];
    if (residual) v += __bfloat162float(residual[m * ldo + n]);
    out[m * ldo + n] = __float2bfloat16_rn(v);
  }
}

// ---- host side -------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::mutex g_encode_mu;

int get_encoder() {
  std::lock_guard<std::mutex> lock(g_encode_mu);
  if (g_encode) return B2F_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
    set_last_cuda_error(e == cudaSuccess ? cudaErrorNotSupported : e);
    return B2F_ERR_CUDA;
  }
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return B2F_OK;
}

// Packed weights of all experts as a 2-D uint32 tensor [E*N rows, K*bits/32
// words]; box = 128 rows x one chunk (8 or 16 words), 32B/64B swizzle.
int make_weight_map(CUtensorMap* map, const uint32_t* w, int64_t rows, int64_t K, int bits) {
  const cuuint64_t words = cuuint64_t(K * bits / 32);
  const cuuint64_t dims[2] = {words, cuuint64_t(rows)};
  const cuuint64_t strides[1] = {words * 4};
  const cuuint32_t box[2] = {cuuint32_t(TC_KC * bits / 32), cuuint32_t(TC_M)};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = bits == 4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(w), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B2F_OK : B2F_ERR_INVALID;
}

template <int BITS, int MAT, int TILE_N>
static int launch_tc_cfg(TcParams p, const CUtensorMap& m0, const CUtensorMap& m1, int64_t slots_grid,
                         cudaStream_t st) {
  constexpr int PK_TILE = TC_M * TC_KC * BITS / 8;
  constexpr int A_TILE = TC_M * TC_KC * 2;
  constexpr int B_TILE = TILE_N * TC_KC * 2;
  // two CTAs per SM when the tiles allow it (each ~110 KB), else one larger CTA
  const int ab_stride = MAT * A_TILE + B_TILE;
  int budget = 108 * 1024;
  if (4 * MAT * PK_TILE + 2 * ab_stride > budget) budget = 200 * 1024;
  int AS = 3, PS = 12;
  while (AS > 2 && 4 * MAT * PK_TILE + AS * ab_stride > budget) --AS;
  while (PS > 2 && PS * MAT * PK_TILE + AS * ab_stride > budget) --PS;
  p.ab_stages = AS;
  p.pk_stages = PS;
  const int smem = 1024 + PS * MAT * PK_TILE + AS * ab_stride + 8 * (2 * PS + 2 * AS + 1) + 32 + 16 * TILE_N;
  if (smem > 227 * 1024) return B2F_ERR_UNSUPPORTED;
  auto kern = qgemm_tc_kernel<BITS, MAT, TILE_N>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return B2F_ERR_CUDA;
  }
  const dim3 grid{unsigned((p.N + TC_M - 1) / TC_M), unsigned(slots_grid), unsigned(p.ksplit)};
  return launch_kernel(kern, grid, dim3{256}, size_t(smem), st, p, m0, m1);
}

template <int BITS, int MAT>
static int launch_tc_bits(const TcParams& p, const CUtensorMap& m0, const CUtensorMap& m1, int64_t slots, int tile,
                          cudaStream_t st) {
  if (tile <= 16) return launch_tc_cfg<BITS, MAT, 16>(p, m0, m1, slots, st);
  if (tile <= 32) return launch_tc_cfg<BITS, MAT, 32>(p, m0, m1, slots, st);
  if (tile <= 64) return launch_tc_cfg<BITS, MAT, 64>(p, m0, m1, slots, st);
  if (tile <= 128) return launch_tc_cfg<BITS, MAT, 128>(p, m0, m1, slots, st);
  return launch_tc_cfg<BITS, MAT, 256>(p, m0, m1, slots, st);
}

static int launch_tc(const TcParams& p, const uint32_t* w0, const uint32_t* w1, int64_t E, int bits, int tile,
                     int64_t slots, cudaStream_t st) {
  int rc = get_encoder();
  if (rc != B2F_OK) return rc;
  CUtensorMap m0, m1;
  rc = make_weight_map(&m0, w0, E * p.N, p.K, bits);
  if (rc != B2F_OK) return rc;
  if (w1) {
    rc = make_weight_map(&m1, w1, E * p.N, p.K, bits);
    if (rc != B2F_OK) return rc;
  } else {
    m1 = m0;
  }
  if (bits == 4) return w1 ? launch_tc_bits<4, 2>(p, m0, m1, slots, tile, st) : launch_tc_bits<4, 1>(p, m0, m1, slots, tile, st);
  return w1 ? launch_tc_bits<8, 2>(p, m0, m1, slots, tile, st) : launch_tc_bits<8, 1>(p, m0, m1, slots, tile, st);
}

static int check_tc_shape(int64_t N, int64_t K, int bits, int gs) {
  if (!(bits == 4 || bits == 8) || gs != 64) return B2F_ERR_UNSUPPORTED;
  if (N <= 0 || K <= 0 || K % 64 != 0) return B2F_ERR_INVALID;
  return B2F_OK;
}

// plan layout helpers live in qgemv.cu
int64_t plan_slots_offset(int64_t A, int64_t E, int tile);
int64_t plan_sorted_offset(int64_t A, int64_t E, int tile);

B2F_DEFINE_WAIT_CONTROLS(tc)

}  // namespace b2f

using namespace b2f;

extern "C" {

int b2f_qgemm_affine_tcgen05(const void* x, int64_t ldx, int64_t M, const uint32_t* wq, const void* scales,
                             const void* biases, int64_t N, int64_t K, int bits, int group_size,
                             const void* residual, void* y, int64_t ldy, int tile, void* stream) {
  int rc = check_tc_shape(N, K, bits, group_size);
  if (rc != B2F_OK) return rc;
  if (M < 0 || tile < 16 || tile > 256 || tile % 16) return B2F_ERR_INVALID;
  if (M == 0) return B2F_OK;
  if (!x || !wq || !scales || !biases || !y) return B2F_ERR_INVALID;
  if (ldx < K || ldy < N) return B2F_ERR_INVALID;
  if (!aligned(x, 16) || (ldx % 8) != 0 || !aligned(wq, 16)) return B2F_ERR_ALIGN;
  TcParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.M = M;
  p.s[0] = static_cast<const __nv_bfloat16*>(scales);
  p.b[0] = static_cast<const __nv_bfloat16*>(biases);
  p.N = N;
  p.K = K;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.out = static_cast<__nv_bfloat16*>(y);
  p.ldo = ldy;
  p.tile = tile;
  p.ksplit = 1;
  const int64_t slots = (M + tile - 1) / tile;
  if (slots > 65535) return B2F_ERR_UNSUPPORTED;
  return launch_tc(p, wq, nullptr, 1, bits, tile, slots, as_stream(stream));
}

int64_t b2f_qgemm_splitk_workspace_bytes(int64_t M, int64_t N, int ksplit) {
  if (M <= 0 || N <= 0 || ksplit <= 0) return 0;
  return int64_t(ksplit) * M * N * int64_t(sizeof(float));
}

int b2f_qgemm_splitk_ranges(int64_t K, int ksplit) {
  if (K <= 0 || K % 64 != 0 || ksplit < 1) return 0;
  const int chunks = int(K / 64);
  const int cps = (chunks + ksplit - 1) / ksplit;
  return (chunks + cps - 1) / cps;
}

int b2f_qgemm_affine_tcgen05_partials(const void* x, int64_t ldx, int64_t M, const uint32_t* wq,
                                      const void* scales, const void* biases, int64_t N, int64_t K, int bits,
                                      int group_size, int tile, int ksplit, float* partial,
                                      int64_t partial_bytes, void* stream) {
  int rc = check_tc_shape(N, K, bits, group_size);
  if (rc != B2F_OK) return rc;
  if (M < 0 || tile < 16 || tile > 256 || tile % 16 || ksplit < 1 || ksplit > 64) return B2F_ERR_INVALID;
  if (M == 0) return B2F_OK;
  if (!x || !wq || !scales || !biases || !partial) return B2F_ERR_INVALID;
  if (ldx < K) return B2F_ERR_INVALID;
  if (!aligned(x, 16) || (ldx % 8) != 0 || !aligned(wq, 16) || !aligned(partial, 16)) return B2F_ERR_ALIGN;
  ksplit = b2f_qgemm_splitk_ranges(K, ksplit);
  if (partial_bytes < b2f_qgemm_splitk_workspace_bytes(M, N, ksplit)) return B2F_ERR_WORKSPACE;
  TcParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.M = M;
  p.s[0] = static_cast<const __nv_bfloat16*>(scales);
  p.b[0] = static_cast<const __nv_bfloat16*>(biases);
  p.N = N;
  p.K = K;
  p.ldo = N;
  p.tile = tile;
  p.ksplit = ksplit;
  p.partial = partial;
  const int64_t slots = (M + tile - 1) / tile;
  if (slots > 65535) return B2F_ERR_UNSUPPORTED;
  return launch_tc(p, wq, nullptr, 1, bits, tile, slots, as_stream(stream));
}

int b2f_qgemm_affine_tcgen05_splitk(const void* x, int64_t ldx, int64_t M, const uint32_t* wq, const void* scales,
                                    const void* biases, int64_t N, int64_t K, int bits, int group_size,
                                    const void* residual, void* y, int64_t ldy, int tile, int ksplit,
                                    void* workspace, int64_t workspace_bytes, void* stream) {
  if (ksplit == 1)
    return b2f_qgemm_affine_tcgen05(x, ldx, M, wq, scales, biases, N, K, bits, group_size, residual, y, ldy, tile,
                                    stream);
  int rc = check_tc_shape(N, K, bits, group_size);
  if (rc != B2F_OK) return rc;
  if (M < 0 || tile < 16 || tile > 256 || tile % 16 || ksplit < 1 || ksplit > 64) return B2F_ERR_INVALID;
  if (M == 0) return B2F_OK;
  if (!x || !wq || !scales || !biases || !y) return B2F_ERR_INVALID;
  if (ldx < K || ldy < N) return B2F_ERR_INVALID;
  if (!aligned(x, 16) || (ldx % 8) != 0 || !aligned(wq, 16)) return B2F_ERR_ALIGN;
  if (!workspace || workspace_bytes < b2f_qgemm_splitk_workspace_bytes(M, N, ksplit)) return B2F_ERR_WORKSPACE;
  if (!aligned(workspace, 16)) return B2F_ERR_ALIGN;
  // every K range non-empty: ksplit ranges of ceil(chunks / ksplit) chunks
  const int chunks = int(K / 64);
  const int cps = (chunks + ksplit - 1) / ksplit;
  ksplit = (chunks + cps - 1) / cps;
  TcParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.M = M;
  p.s[0] = static_cast<const __nv_bfloat16*>(scales);
  p.b[0] = static_cast<const __nv_bfloat16*>(biases);
  p.N = N;
  p.K = K;
  p.out = static_cast<__nv_bfloat16*>(y);
  p.ldo = ldy;
  p.tile = tile;
  p.ksplit = ksplit;
  p.partial = static_cast<float*>(workspace);
  const int64_t slots = (M + tile - 1) / tile;
  if (slots > 65535) return B2F_ERR_UNSUPPORTED;
  cudaStream_t st = as_stream(stream);
  rc = launch_tc(p, wq, nullptr, 1, bits, tile, slots, st);
  if (rc != B2F_OK) return rc;
  const int64_t total = M * N;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (total + 255) / 256;
  return launch_kernel(splitk_finalize_kernel, dim3{unsigned(blocks < int64_t(sms) * 8 ? blocks : int64_t(sms) * 8)},
                       dim3{256}, 0, st, static_cast<const float*>(p.partial), int(ksplit), int64_t(M), int64_t(N),
                       static_cast<const __nv_bfloat16*>(residual), p.out, int64_t(ldy));
}

int b2f_gather_qgemm_affine_tcgen05(const void* x, int64_t ldx, const int32_t* x_row_index, int64_t x_row_div,
                                    int64_t A, int64_t E, const uint32_t* w_gate, const void* s_gate,
                                    const void* b_gate, const uint32_t* w_up, const void* s_up, const void* b_up,
                                    int64_t N, int64_t K, int bits, int group_size, int tile,
                                    const void* plan_workspace, int64_t plan_workspace_bytes, void* out, int64_t ldo,
                                    void* stream) {
  int rc = check_tc_shape(N, K, bits, group_size);
  if (rc != B2F_OK) return rc;
  if (A < 0 || E <= 0 || tile < 16 || tile > 256 || tile % 16) return B2F_ERR_INVALID;
  if (A == 0) return B2F_OK;
  if (!x || !w_gate || !s_gate || !b_gate || !out) return B2F_ERR_INVALID;
  if (w_up && (!s_up || !b_up)) return B2F_ERR_INVALID;
  if (!x_row_index && x_row_div <= 0) return B2F_ERR_INVALID;
  if (ldx < K || ldo < N) return B2F_ERR_INVALID;
  if (!aligned(x, 16) || (ldx % 8) != 0 || !aligned(w_gate, 16) || (w_up && !aligned(w_up, 16)))
    return B2F_ERR_ALIGN;
  const int64_t need = b2f_moe_plan_workspace_bytes(A, E, tile);
  if (!plan_workspace || plan_workspace_bytes < need) return B2F_ERR_WORKSPACE;
  const char* ws = static_cast<const char*>(plan_workspace);
  TcParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.x_row_index = x_row_index;
  p.x_row_div = x_row_div > 0 ? x_row_div : 1;
  p.ksplit = 1;
  p.s[0] = static_cast<const __nv_bfloat16*>(s_gate);
  p.b[0] = static_cast<const __nv_bfloat16*>(b_gate);
  p.s[1] = static_cast<const __nv_bfloat16*>(s_up);
  p.b[1] = static_cast<const __nv_bfloat16*>(b_up);
  p.sb_estride = N * (K / group_size);
  p.N = N;
  p.K = K;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.slot_count = reinterpret_cast<const int32_t*>(ws);
  // a bounded wait that gives up records B2F_ERR_TIMEOUT in the plan header's status word
  p.err = const_cast<int32_t*>(reinterpret_cast<const int32_t*>(ws)) + 1;
  p.slots = reinterpret_cast<const int4*>(ws + plan_slots_offset(A, E, tile));
  p.sorted = reinterpret_cast<const int32_t*>(ws + plan_sorted_offset(A, E, tile));
  p.tile = tile;
  const int64_t max_slots = b2f_moe_plan_max_slots(A, E, tile);
  if (max_slots > 65535) return B2F_ERR_UNSUPPORTED;
  return launch_tc(p, w_gate, w_up, E, bits, tile, max_slots, as_stream(stream));
}

}  // extern "C"
