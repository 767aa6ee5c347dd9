// (c) grouped expert GEMM on tcgen05/TMEM over expert-sorted token rows.
//
// The MoE plan (plan.cuh) orders the routed assignments by expert.  With
// the activations copied into that order once per layer (b2f_moe_gather_rows,
// which also applies the K order the weight unpack produces), every token
// tile of an expert is a run of consecutive rows, so the tile's x block for a
// K-chunk is one 2-D TMA load straight into the 128B-swizzled MMA layout.
// The gate/up call writes its output rows in the same sorted, K-permuted
// layout, so the down projection reads them the same way; the down call
// writes rows back in assignment order for the weighted combine.
//
// Persistent CTAs (one per SM) walk the work units (slot, 128-row block) of
// the plan; the pipeline runs across unit boundaries:
//   warp 0      producer: per stage of SC K-chunks one TMA load of the
//               packed words per matrix (SC*32 or SC*64 bytes per row, so a
//               stage moves whole 128-byte row segments) and the x tiles of
//               those chunks, 16 token rows per load and only as many rows
//               as the slot has, into a PS-deep ring.
//   warp 1      MMA issuer (one thread): tcgen05.mma kind::f16, bf16 x bf16
//               -> fp32 TMEM accumulators; tcgen05.commit frees stages.
//   warps 2-9   converters: thread (row, K half) dequantizes 32 values of its
//               row, w = q*s + b in one bf16 rounding, into the AS-deep A
//               ring; then the epilogue (TMEM -> registers -> bf16 rows).
//               Scales and biases come in blocks of 8 groups (4-byte loads
//               into registers), one block ahead in the CTA's unit order,
//               so their memory latency hides behind 8 chunks of work.
// Every wait is bounded: on a timeout the kernel records B2F_ERR_TIMEOUT,
// drains its own copies and MMAs (bounded), frees TMEM and returns.
#include "common.cuh"
#include "plan.cuh"
#include "tc_common.cuh"

namespace b2f {

constexpr int TC2_THREADS = 320;
constexpr int TC2_CONV_WARPS = 8;
constexpr int TC2_SB_CHUNKS = 8;  // chunks per scale/bias register block

struct Tc2Params {
  const int32_t* slot_count;
  const int4* slots;
  const int32_t* sorted;
  const __nv_bfloat16* s[2];
  const __nv_bfloat16* b[2];
  int64_t sb_estride;  // scale elements per expert matrix (N * K/64)
  int64_t N, K;
  __nv_bfloat16* out;
  int64_t ldo;
  int out_sorted;
  int n_rb;
  int max_slots;
  int32_t* err;
  int PS, AS;
};

// Position of K index k inside its group of 8 in the permuted layout
// (0,4,1,5,2,6,3,7): the order the nibble unpack emits pairs in.
__device__ __forceinline__ int64_t kperm_col(int64_t k) { return (k & ~int64_t(7)) | ((k & 3) << 1) | ((k >> 2) & 1); }

template <int BITS, int MAT, int TILE_N, int SC>
__global__ void __launch_bounds__(TC2_THREADS, 1) qgemm_tc2_kernel(const Tc2Params p,
                                                                  const __grid_constant__ CUtensorMap tmx,
                                                                  const __grid_constant__ CUtensorMap tm0,
                                                                  const __grid_constant__ CUtensorMap tm1) {
  constexpr int PKB = TC_KC * BITS / 8;  // packed bytes per row per chunk
  constexpr int PITCH = SC * PKB;        // packed bytes per row per stage
  constexpr int PK_TILE = TC_M * PITCH;  // per matrix per stage
  constexpr int A_TILE = TC_M * TC_KC * 2;
  constexpr int B_TILE = TILE_N * TC_KC * 2;  // per chunk
  constexpr int STAGE = SC * B_TILE + MAT * PK_TILE;
  constexpr uint32_t TMEM_COLS = (MAT * TILE_N <= 32) ? 32 : (MAT * TILE_N <= 64) ? 64 : (MAT * TILE_N <= 128) ? 128
                                 : (MAT * TILE_N <= 256) ? 256 : 512;
  constexpr int PK_SW_MASK = PITCH / 16 - 1;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int PS = p.PS, AS = p.AS;

  uint8_t* stages = smem;                              // [PS][SC B tiles | MAT pk tiles]
  uint8_t* atiles = stages + PS * STAGE;               // [AS][MAT][A_TILE]
  uint64_t* bars = reinterpret_cast<uint64_t*>(atiles + AS * MAT * A_TILE);
  uint64_t* full = bars;
  uint64_t* empty = full + PS;
  uint64_t* a_full = empty + PS;
  uint64_t* a_empty = a_full + AS;
  uint64_t* acc_full = a_empty + AS;
  uint64_t* drain = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if (tid == 0) {
    for (int s = 0; s < PS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < AS; ++s) {
      mbar_init(&a_full[s], TC2_CONV_WARPS);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int n_slots = *p.slot_count;
  if (n_slots > p.max_slots) n_slots = p.max_slots;
  const int n_units = n_slots * p.n_rb;
  const int n_chunks = int(p.K / TC_KC);
  const int64_t ngroups = p.K / TC_KC;

  if (warp == 0) {
    // =============================== producer ===================================
    // Control flow stays warp-uniform: lane 0 waits, the verdict is broadcast.
    int gsx = 0;  // stage sequence number
    bool stop = __shfl_sync(0xffffffffu, *abort_flag, 0) != 0;
    const bool stall = producers_stalled();  // test control: nothing is issued
    for (int u = blockIdx.x; u < n_units && !stop && !stall; u += gridDim.x) {
      const int4 sl = p.slots[u / p.n_rb];
      const int64_t m0 = int64_t(u % p.n_rb) * TC_M;
      const int row0 = int(int64_t(sl.x) * p.N + m0);
      const int n16 = (sl.z + 15) >> 4;  // 16-row x boxes per chunk
      for (int c0 = 0; c0 < n_chunks; c0 += SC) {
        int ok = 1;
        if (lane == 0) {
          const int s = gsx % PS;
          ok = !*abort_flag && (gsx < PS || mbar_wait_bounded(&empty[s], uint32_t(((gsx / PS) - 1) & 1)));
          if (ok) {
            const int nsub = min(SC, n_chunks - c0);
            uint8_t* st = stages + s * STAGE;
            mbar_arrive_expect_tx(&full[s], uint32_t(MAT * PK_TILE + nsub * n16 * 16 * TC_KC * 2));
            tma_load_2d(st + SC * B_TILE, &tm0, (c0 / SC) * (PITCH / 4), row0, &full[s]);
            if constexpr (MAT == 2) tma_load_2d(st + SC * B_TILE + PK_TILE, &tm1, (c0 / SC) * (PITCH / 4), row0, &full[s]);
            for (int cc = 0; cc < nsub; ++cc)
              for (int r = 0; r < n16; ++r)
                tma_load_2d(st + cc * B_TILE + r * 16 * TC_KC * 2, &tmx, (c0 + cc) * TC_KC, sl.y + 16 * r, &full[s]);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          stop = true;
          break;
        }
        ++gsx;
      }
    }
    if (stop && lane == 0) *abort_flag = 1;
    if (lane == 0 && stop) {
      // let the TMA loads already issued land before the CTA goes away
      for (int k = 1; k <= PS && gsx - k >= 0; ++k) {
        const int gi = gsx - k;
        mbar_wait_bounded(&full[gi % PS], uint32_t((gi / PS) & 1), 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // =============================== MMA issuer =================================
    if (lane == 0) {
      int g = 0, gsx = 0;
      for (int u = blockIdx.x; u < n_units && !*abort_flag; u += gridDim.x) {
        const int4 sl = p.slots[u / p.n_rb];
        const int n_pad = (sl.z + 15) & ~15;
        const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n_pad >> 3) << 17) |
                               (uint32_t(TC_M >> 4) << 24);
        for (int c = 0; c < n_chunks; ++c, ++g) {
          const int s = gsx % PS, sa = g % AS, cc = c % SC;
          if (!mbar_wait_bounded(&full[s], uint32_t((gsx / PS) & 1)) ||
              !mbar_wait_bounded(&a_full[sa], uint32_t((g / AS) & 1))) {
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = sw128_desc(stages + s * STAGE + cc * B_TILE);
#pragma unroll
          for (int m = 0; m < MAT; ++m) {
            const uint64_t adesc = sw128_desc(atiles + (sa * MAT + m) * A_TILE);
#pragma unroll
            for (int ks = 0; ks < TC_KC / 16; ++ks)
              tc_mma(tmem + uint32_t(m * TILE_N), adesc + 2 * ks, bdesc + 2 * ks, idesc,
                     (c > 0 || ks > 0) ? 1u : 0u);
          }
          tc_commit(&a_empty[sa]);
          if (cc == SC - 1 || c == n_chunks - 1) {
            tc_commit(&empty[s]);
            ++gsx;
          }
          if (c == n_chunks - 1) tc_commit(acc_full);
        }
      }
      // all MMAs issued by this thread complete before TMEM is released
      tc_commit(drain);
      mbar_wait_bounded(drain, 0u, 100000000ull);
    }
    __syncwarp();
  } else {
    // =============================== converters / epilogue ========================
    const int tc = tid - 64;          // 0..255
    const int t = tc & (TC_M - 1);    // row within the block
    const int h = tc >> 7;            // K half of the chunk
    const int sw = (t * PITCH >> 7) & PK_SW_MASK;  // TMA swizzle of this packed row
    // Every lane waits on the barriers; the verdict is made warp-uniform
    // (__all_sync) so the .sync.aligned TMEM loads and __syncwarp never diverge.
    // scale/bias register blocks: [m][s|b][4 words = 8 groups]; `nxt` is
    // loaded one block ahead along this CTA's (unit, block) sequence
    const int nblk = (n_chunks + TC2_SB_CHUNKS - 1) / TC2_SB_CHUNKS;
    uint32_t cur[MAT][2][4], nxt[MAT][2][4];
    int pu = blockIdx.x, pj = 0;
    auto load_block = [&](uint32_t (&dst)[MAT][2][4]) {
      const bool live = pu < n_units;
      int64_t base = 0;
      int64_t row = TC_M;
      if (live) {
        const int4 su = p.slots[pu / p.n_rb];
        row = int64_t(pu % p.n_rb) * TC_M + t;
        base = int64_t(su.x) * p.sb_estride + row * ngroups + int64_t(pj) * TC2_SB_CHUNKS;
      }
#pragma unroll
      for (int m = 0; m < MAT; ++m)
#pragma unroll
        for (int kind = 0; kind < 2; ++kind) {
          const __nv_bfloat16* src = kind ? (m ? p.b[1] : p.b[0]) : (m ? p.s[1] : p.s[0]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int64_t gg = int64_t(pj) * TC2_SB_CHUNKS + 2 * i;
            dst[m][kind][i] = (live && row < p.N && gg < ngroups)
                                  ? __ldg(reinterpret_cast<const uint32_t*>(src + base + 2 * i))
                                  : 0u;
          }
        }
      if (++pj == nblk) {
        pj = 0;
        pu += gridDim.x;
      }
    };
    load_block(cur);
    load_block(nxt);
    int g = 0, it = 0, gsx = 0;
    bool stop = __shfl_sync(0xffffffffu, *abort_flag, 0) != 0;
    for (int u = blockIdx.x; u < n_units && !stop; u += gridDim.x, ++it) {
      const int4 sl = p.slots[u / p.n_rb];
      const int64_t m0 = int64_t(u % p.n_rb) * TC_M;
      for (int c = 0; c < n_chunks; ++c, ++g) {
        const int s = gsx % PS, sa = g % AS, cc = c % SC;
        if (c % TC2_SB_CHUNKS == 0 && g > 0) {
#pragma unroll
          for (int m = 0; m < MAT; ++m)
#pragma unroll
            for (int kind = 0; kind < 2; ++kind)
#pragma unroll
              for (int i = 0; i < 4; ++i) cur[m][kind][i] = nxt[m][kind][i];
          load_block(nxt);
        }
        const bool ok = !(*abort_flag) && mbar_wait_bounded(&full[s], uint32_t((gsx / PS) & 1)) &&
                        (g < AS || mbar_wait_bounded(&a_empty[sa], uint32_t(((g / AS) - 1) & 1)));
        if (!__all_sync(0xffffffffu, ok)) {
          stop = true;
          break;
        }
        const int cw = (c % TC2_SB_CHUNKS) >> 1, chi = c & 1;  // word and half of this chunk's group
#pragma unroll
        for (int m = 0; m < MAT; ++m) {
          const uint32_t sw4 = cw == 0 ? cur[m][0][0] : cw == 1 ? cur[m][0][1] : cw == 2 ? cur[m][0][2] : cur[m][0][3];
          const uint32_t bw4 = cw == 0 ? cur[m][1][0] : cw == 1 ? cur[m][1][1] : cw == 2 ? cur[m][1][2] : cur[m][1][3];
          // broadcast the chunk's bf16 (low half = even group) to both halves
          const uint32_t s2v = prmt(sw4, 0u, chi ? 0x3232u : 0x1010u);
          const uint32_t b2v = prmt(bw4, 0u, chi ? 0x3232u : 0x1010u);
          const uint8_t* prow = stages + s * STAGE + SC * B_TILE + m * PK_TILE + t * PITCH;
          uint8_t* arow = atiles + (sa * MAT + m) * A_TILE;
          if constexpr (BITS == 4) {
            // this thread's 16 B = 4 words = K values 32h .. 32h+31
            const uint4 q = *reinterpret_cast<const uint4*>(prow + (((2 * cc + h) ^ sw) << 4));
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
          } else {
            // 32 B = two 16-byte pieces 2h, 2h+1; words (2i, 2i+1) -> A chunk i
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int piece = 2 * h + hh;
              const uint4 q = *reinterpret_cast<const uint4*>(prow + (((4 * cc + piece) ^ sw) << 4));
              const uint32_t wds[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
              for (int ii = 0; ii < 2; ++ii) {
                const uint32_t wa = wds[2 * ii], wb = wds[2 * ii + 1];
                uint32_t o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float qa = float((wa >> (8 * j)) & 0xFFu), qb = float((wb >> (8 * j)) & 0xFFu);
                  o[j] = hfma2_bf(pack_bf16x2(qa, qb), s2v, b2v);
                }
                *reinterpret_cast<uint4*>(arow + sw128_off(t, 2 * piece + ii)) = make_uint4(o[0], o[1], o[2], o[3]);
              }
            }
          }
        }
        fence_proxy_async_smem();  // generic stores -> tensor-core reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
        if (cc == SC - 1 || c == n_chunks - 1) ++gsx;
      }
      if (stop) break;
      // ---- epilogue: TMEM -> registers -> bf16 ---------------------------------
      if (!__all_sync(0xffffffffu, !(*abort_flag) && mbar_wait_bounded(acc_full, uint32_t(it & 1)))) {
        stop = true;
        break;
      }
      tc_fence_after();
      const int qd = warp & 3;           // TMEM lane quarter this warp may read
      const int ch = (warp - 2) >> 2;    // which 16-column blocks
      const int row = 32 * qd + lane;
      const int64_t gr = m0 + row;
      const int n_tok = sl.z, n_pad = (n_tok + 15) & ~15;
      const int64_t col = p.out_sorted ? kperm_col(gr) : gr;
      for (int n0 = 16 * ch; n0 < n_pad; n0 += 32) {
        uint32_t gv[16], uv[16];
        tmem_ld16(tmem + (uint32_t(32 * qd) << 16) + uint32_t(n0), gv);
        if constexpr (MAT == 2) tmem_ld16(tmem + (uint32_t(32 * qd) << 16) + uint32_t(TILE_N + n0), uv);
        if (gr < p.N) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = n0 + i;
            if (n < n_tok) {
              float v = __uint_as_float(gv[i]);
              if constexpr (MAT == 2) v = silu_mul_tc(v, __uint_as_float(uv[i]));
              const int64_t o = p.out_sorted ? int64_t(sl.y + n) : int64_t(p.sorted[sl.y + n]);
              p.out[o * p.ldo + col] = __float2bfloat16_rn(v);
            }
          }
        }
      }
      tc_fence_before();  // TMEM reads ordered before the next unit's MMAs
    }
    if (stop && lane == 0) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
  if (tid == 0 && *abort_flag) report_timeout(p.err);
}

// out[i, :] = x[row(sorted[i]), :] for every planned assignment i, each group
// of 8 columns permuted to (0,4,1,5,2,6,3,7).
__global__ void __launch_bounds__(256) moe_gather_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                              const int32_t* __restrict__ x_row_index,
                                                              int64_t x_row_div, const int32_t* __restrict__ sorted,
                                                              const int32_t* __restrict__ total_ptr, int64_t K,
                                                              __nv_bfloat16* __restrict__ out, int64_t ldo,
                                                              int64_t A) {
  const int64_t total = min(int64_t(*total_ptr), A);
  const int64_t vpr = K / 8;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total * vpr;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = idx / vpr, v = idx - i * vpr;
    const int a = sorted[i];
    const int64_t xr = x_row_index ? int64_t(x_row_index[a]) : int64_t(a) / x_row_div;
    const uint4 xv = *reinterpret_cast<const uint4*>(x + xr * ldx + 8 * v);
    *reinterpret_cast<uint4*>(out + i * ldo + 8 * v) =
        make_uint4(prmt(xv.x, xv.z, 0x5410u), prmt(xv.x, xv.z, 0x7632u), prmt(xv.y, xv.w, 0x5410u),
                   prmt(xv.y, xv.w, 0x7632u));
  }
}

static int make_rows_map(CUtensorMap* map, const void* x, int64_t rows, int64_t K, int64_t ldx, int box_rows) {
  const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ldx) * 2};
  const cuuint32_t box[2] = {cuuint32_t(TC_KC), cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B2F_OK : B2F_ERR_INVALID;
}

static int g_sms_tc2 = 0;

// Packed weights as a 2-D uint32 tensor [rows, K*bits/32 words]; box = 128
// rows x `pitch` bytes (SC chunks), swizzle matching the pitch.
static int make_weight_map_pitch(CUtensorMap* map, const uint32_t* w, int64_t rows, int64_t K, int bits,
                                 int pitch) {
  const cuuint64_t words = cuuint64_t(K * bits / 32);
  const cuuint64_t dims[2] = {words, cuuint64_t(rows)};
  const cuuint64_t strides[1] = {words * 4};
  const cuuint32_t box[2] = {cuuint32_t(pitch / 4), cuuint32_t(TC_M)};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = pitch == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : pitch == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                              : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(w), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B2F_OK : B2F_ERR_INVALID;
}

struct Tc2Maps {
  const void* x;
  int64_t x_rows, ldx;
  const uint32_t* w0;
  const uint32_t* w1;
  int64_t w_rows;
};

// Stages and A-ring depth for a configuration; false if PS < 2.
template <int BITS, int MAT, int TILE_N, int SC>
static bool tc2_plan(int* PS_out, int* AS_out, int* smem_out) {
  constexpr int PITCH = SC * TC_KC * BITS / 8;
  constexpr int PK_TILE = TC_M * PITCH;
  constexpr int A_TILE = TC_M * TC_KC * 2;
  constexpr int B_TILE = TILE_N * TC_KC * 2;
  constexpr int STAGE = SC * B_TILE + MAT * PK_TILE;
  const int budget = 220 * 1024;
  int AS = 3;
  if (MAT * A_TILE * AS + 3 * STAGE > budget) AS = 2;
  int PS = (budget - AS * MAT * A_TILE - 1024 - 256) / STAGE;
  if (PS > 8) PS = 8;
  *PS_out = PS;
  *AS_out = AS;
  *smem_out = 1024 + PS * STAGE + AS * MAT * A_TILE + 8 * (2 * PS + 2 * AS + 2) + 16;
  return PS >= 2 && *smem_out <= 227 * 1024;
}

template <int BITS, int MAT, int TILE_N, int SC>
static int launch_tc2_cfg(Tc2Params p, const Tc2Maps& maps, cudaStream_t st) {
  int PS, AS, smem;
  if (!tc2_plan<BITS, MAT, TILE_N, SC>(&PS, &AS, &smem)) return B2F_ERR_UNSUPPORTED;
  p.PS = PS;
  p.AS = AS;
  CUtensorMap mx, m0, m1;
  int rc = make_rows_map(&mx, maps.x, maps.x_rows, p.K, maps.ldx, 16);
  if (rc != B2F_OK) return rc;
  constexpr int PITCH = SC * TC_KC * BITS / 8;
  rc = make_weight_map_pitch(&m0, maps.w0, maps.w_rows, p.K, BITS, PITCH);
  if (rc != B2F_OK) return rc;
  if (maps.w1) {
    rc = make_weight_map_pitch(&m1, maps.w1, maps.w_rows, p.K, BITS, PITCH);
    if (rc != B2F_OK) return rc;
  } else {
    m1 = m0;
  }
  auto kern = qgemm_tc2_kernel<BITS, MAT, TILE_N, SC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return B2F_ERR_CUDA;
  }
  if (g_sms_tc2 == 0) {
    int dev = 0, n = 0;
    g_sms_tc2 = (cudaGetDevice(&dev) == cudaSuccess &&
                 cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
                    ? n
                    : 148;
  }
  const int64_t max_units = int64_t(p.max_slots) * p.n_rb;
  const int grid = int(max_units < g_sms_tc2 ? max_units : g_sms_tc2);
  kern<<<grid < 1 ? 1 : grid, TC2_THREADS, smem, st>>>(p, mx, m0, m1);
  return check_launch();
}

// Widest stage (most chunks per weight load) that still leaves >= 3 stages,
// else the widest with >= 2.
template <int BITS, int MAT, int TILE_N>
static int launch_tc2_tile(const Tc2Params& p, const Tc2Maps& maps, cudaStream_t st) {
  int PS, AS, smem;
  if constexpr (BITS == 4) {
    if (tc2_plan<4, MAT, TILE_N, 4>(&PS, &AS, &smem) && PS >= 3) return launch_tc2_cfg<4, MAT, TILE_N, 4>(p, maps, st);
  }
  if (tc2_plan<BITS, MAT, TILE_N, 2>(&PS, &AS, &smem) && PS >= 3) return launch_tc2_cfg<BITS, MAT, TILE_N, 2>(p, maps, st);
  if (tc2_plan<BITS, MAT, TILE_N, 1>(&PS, &AS, &smem) && PS >= 3) return launch_tc2_cfg<BITS, MAT, TILE_N, 1>(p, maps, st);
  if constexpr (BITS == 4) {
    if (tc2_plan<4, MAT, TILE_N, 4>(&PS, &AS, &smem)) return launch_tc2_cfg<4, MAT, TILE_N, 4>(p, maps, st);
  }
  if (tc2_plan<BITS, MAT, TILE_N, 2>(&PS, &AS, &smem)) return launch_tc2_cfg<BITS, MAT, TILE_N, 2>(p, maps, st);
  return launch_tc2_cfg<BITS, MAT, TILE_N, 1>(p, maps, st);
}

template <int BITS, int MAT>
static int launch_tc2_bits(const Tc2Params& p, const Tc2Maps& maps, int tile, cudaStream_t st) {
  if (tile <= 16) return launch_tc2_tile<BITS, MAT, 16>(p, maps, st);
  if (tile <= 32) return launch_tc2_tile<BITS, MAT, 32>(p, maps, st);
  if (tile <= 64) return launch_tc2_tile<BITS, MAT, 64>(p, maps, st);
  if (tile <= 128) return launch_tc2_tile<BITS, MAT, 128>(p, maps, st);
  return launch_tc2_tile<BITS, MAT, 256>(p, maps, st);
}

B2F_DEFINE_WAIT_CONTROLS(tc2)

}  // namespace b2f

using namespace b2f;

extern "C" {

int b2f_moe_gather_rows(const void* x, int64_t ldx, const int32_t* x_row_index, int64_t x_row_div, int64_t A,
                        int64_t E, int tile, const void* plan_workspace, int64_t plan_workspace_bytes, int64_t K,
                        void* out, int64_t ldo, void* stream) {
  if (A < 0 || E <= 0 || K <= 0 || K % 8 != 0 || ldx < K || ldo < K) return B2F_ERR_INVALID;
  if (!x_row_index && x_row_div <= 0) return B2F_ERR_INVALID;
  if (A == 0) return B2F_OK;
  if (!x || !out || !plan_workspace) return B2F_ERR_INVALID;
  if (!aligned(x, 16) || !aligned(out, 16) || ldx % 8 || ldo % 8) return B2F_ERR_ALIGN;
  const PlanLayout L = plan_layout(A, E, tile);
  if (plan_workspace_bytes < L.total) return B2F_ERR_WORKSPACE;
  const char* ws = static_cast<const char*>(plan_workspace);
  const int32_t* offsets = reinterpret_cast<const int32_t*>(ws + L.off_offsets);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t work = A * (K / 8);
  const int64_t blocks = (work + 255) / 256;
  const int grid = int(blocks < int64_t(sms) * 8 ? blocks : int64_t(sms) * 8);
  moe_gather_rows_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, x_row_index, x_row_div > 0 ? x_row_div : 1,
      reinterpret_cast<const int32_t*>(ws + L.off_sorted), offsets + E, K, static_cast<__nv_bfloat16*>(out), ldo, A);
  return check_launch();
}

int b2f_sorted_qgemm_affine_tcgen05(const void* x_sorted, int64_t ldx, int64_t A, int64_t E, const uint32_t* w_gate,
                                    const void* s_gate, const void* b_gate, const uint32_t* w_up, const void* s_up,
                                    const void* b_up, int64_t N, int64_t K, int bits, int group_size, int tile,
                                    const void* plan_workspace, int64_t plan_workspace_bytes, void* out, int64_t ldo,
                                    int out_sorted, void* stream) {
  if (!(bits == 4 || bits == 8) || group_size != 64) return B2F_ERR_UNSUPPORTED;
  if (N <= 0 || K <= 0 || K % 64 != 0) return B2F_ERR_INVALID;
  if ((K / 64) % 2 != 0) return B2F_ERR_UNSUPPORTED;  // 4-byte scale loads cover two groups
  if (A < 0 || E <= 0 || tile < 16 || tile > 256 || tile % 16) return B2F_ERR_INVALID;
  if (A == 0) return B2F_OK;
  if (!x_sorted || !w_gate || !s_gate || !b_gate || !out || !plan_workspace) return B2F_ERR_INVALID;
  if (out_sorted && N % 8 != 0) return B2F_ERR_INVALID;  // permuted columns stay inside the row
  if (w_up && (!s_up || !b_up)) return B2F_ERR_INVALID;
  if (ldx < K || ldo < N) return B2F_ERR_INVALID;
  if (!aligned(x_sorted, 16) || ldx % 8 || !aligned(w_gate, 16) || (w_up && !aligned(w_up, 16)))
    return B2F_ERR_ALIGN;
  if (!aligned(s_gate, 4) || !aligned(b_gate, 4) || (w_up && (!aligned(s_up, 4) || !aligned(b_up, 4))))
    return B2F_ERR_ALIGN;
  const PlanLayout L = plan_layout(A, E, tile);
  if (plan_workspace_bytes < L.total) return B2F_ERR_WORKSPACE;
  const int64_t max_slots = plan_max_slots(A, E, tile);
  const int64_t n_rb = (N + TC_M - 1) / TC_M;
  if (max_slots * n_rb > 0x7fffffff || E * N > 0x7fffffff || A > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  const char* ws = static_cast<const char*>(plan_workspace);
  Tc2Params p{};
  p.slot_count = reinterpret_cast<const int32_t*>(ws + L.off_hdr);
  // a bounded wait that gives up records B2F_ERR_TIMEOUT in the plan header's status word
  p.err = const_cast<int32_t*>(reinterpret_cast<const int32_t*>(ws + L.off_hdr)) + 1;
  p.slots = reinterpret_cast<const int4*>(ws + L.off_slots);
  p.sorted = reinterpret_cast<const int32_t*>(ws + L.off_sorted);
  p.s[0] = static_cast<const __nv_bfloat16*>(s_gate);
  p.b[0] = static_cast<const __nv_bfloat16*>(b_gate);
  p.s[1] = static_cast<const __nv_bfloat16*>(w_up ? s_up : s_gate);
  p.b[1] = static_cast<const __nv_bfloat16*>(w_up ? b_up : b_gate);
  p.sb_estride = N * (K / 64);
  p.N = N;
  p.K = K;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.out_sorted = out_sorted ? 1 : 0;
  p.n_rb = int(n_rb);
  p.max_slots = int(max_slots);
  int rc = get_encoder();
  if (rc != B2F_OK) return rc;
  Tc2Maps maps{x_sorted, A, ldx, w_gate, w_up, E * N};
  cudaStream_t st = as_stream(stream);
  if (bits == 4) return w_up ? launch_tc2_bits<4, 2>(p, maps, tile, st) : launch_tc2_bits<4, 1>(p, maps, tile, st);
  return w_up ? launch_tc2_bits<8, 2>(p, maps, tile, st) : launch_tc2_bits<8, 1>(p, maps, tile, st);
}

}  // extern "C"
