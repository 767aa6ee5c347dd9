// (d) paged decode attention that reads the reference KV format directly
// (uint8 codes + float32 per-64 scales, quantized_kv_cache.py:68-156): one
// query token per sequence, grouped-query heads sharing each KV head.
//
// Layout in HBM (per layer):
//   K/V codes  uint8 [num_pages][Hkv][page][D*bits/8]   (one reference row per token)
//   K/V scales f32   [num_pages][Hkv][page][D/64]
//   block_table int32 [B][max_pages], seq_lens int32 [B]
// A CTA = (split of the context, kv head, sequence); 4 warps walk 16-token
// sub-tiles of the split.  Per sub-tile:
//   S = Q.K^T   warp MMA m16n8k16 (fp16 in, fp32 acc): rows = the G query
//               heads of this KV head, k = head_dim, n = 8 tokens.  K codes
//               become fp16 1024+code with one prmt/lop3 per two values;
//               per 64-wide group: s += kscale*(acc - (1024+max_int)*sum(q))
//   online softmax in base 2 (q is pre-scaled by softmax_scale*log2(e))
//   O += P.V    P from the S accumulators (FA2 register reuse), V codes
//               decoded to fp16 (code-max_int)*vscale in registers.
// Splits write (m, l, O) partials; a combine kernel merges them.
#include "common.cuh"
#include "tc_common.cuh"

namespace b2f {

struct AttnParams {
  const __nv_bfloat16* q;
  const uint8_t* kp;
  const float* ks;
  const uint8_t* vp;
  const float* vs;
  const int32_t* block_table;
  int64_t max_pages;
  const int32_t* seq_lens;
  int B, Hq, Hkv, G, PS, n_splits;
  int64_t head_stride, slot_stride;  // rows between heads / between slots of a page
  float qscale;
  float* o_part;
  float* ml_part;
  __nv_bfloat16* out;
  int ring_bytes;  // ring path: shared-memory bytes of the page ring (the merge area follows)
  int slot_bytes;  // ring path: bytes of one ring slot
};

// Named barrier `id` over the first `n` threads of the CTA.
__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

constexpr int ATTN_RING = 4;  // pages in flight per CTA on the ring path

// Byte offset of `byte` of K/V code row `row` inside a TMA tile of rows of
// RB bytes written with the swizzle matching RB (128B / 64B / 32B).
template <int RB>
__device__ __forceinline__ int swz_off(int row, int byte) {
  constexpr int MASK = RB / 16 - 1;
  const int sw = ((row * RB) >> 7) & MASK;
  return row * RB + ((((byte >> 4) ^ sw)) << 4) + (byte & 15);
}

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }

template <int BITS, int D, bool RING>
__global__ void __launch_bounds__(RING ? 160 : 128) qkv_decode_attn_kernel(const AttnParams p,
                                                                         const __grid_constant__ CUtensorMap tmk,
                                                                         const __grid_constant__ CUtensorMap tmv) {
  pdl_enter();
  constexpr int DG = D / 64;      // quantization groups per row
  constexpr int KSTEPS = D / 16;  // MMA k-steps for Q.K^T
  constexpr int NTD = D / 8;      // 8-wide output column tiles
  constexpr int RB = D * BITS / 8;
  constexpr float MI = BITS == 8 ? 127.f : BITS == 4 ? 7.f : 1.f;
  constexpr float KOFF = 1024.f + MI;
  constexpr int KW = BITS == 8 ? 4 : BITS == 4 ? 2 : 1;  // K words per thread per group per token
  constexpr int VW = BITS == 8 ? 2 : 1;                  // V words per thread per group per token

  const int split = blockIdx.x, hkv = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int G = p.G;
  const int len = p.seq_lens[b];
  const int n_sub = (len + 15) / 16;
  const int per_split = (n_sub + p.n_splits - 1) / p.n_splits;
  const int sub_begin = split * per_split;
  const int sub_end = min(n_sub, sub_begin + per_split);

  // ---- Q fragments (fp16, pre-scaled) and per-group sums of q -----------
  uint32_t qa[KSTEPS][4];
  float qg[2][DG];
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    const int head = r + 8 * h2;
    const bool hv = head < G;
    const __nv_bfloat16* qrow = p.q + (int64_t(b) * p.Hq + int64_t(hkv) * G + head) * D;
#pragma unroll
    for (int g = 0; g < DG; ++g) {
      float v[16];
      if (hv) {
        const uint4* src = reinterpret_cast<const uint4*>(qrow + 64 * g + 16 * c);
        const uint4 a = src[0], bb = src[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, bb.x, bb.y, bb.z, bb.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
          v[2 * i] = round_f16(__low2float(h) * p.qscale);
          v[2 * i + 1] = round_f16(__high2float(h) * p.qscale);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
      }
      float part = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) part += v[i];
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      qg[h2][g] = part;
      if constexpr (BITS == 8) {
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          qa[g * 4 + s][h2] = pack_f16x2(v[4 * s], v[4 * s + 1]);
          qa[g * 4 + s][2 + h2] = pack_f16x2(v[4 * s + 2], v[4 * s + 3]);
        }
      } else if constexpr (BITS == 2) {
        // k-step st takes the crumb pairs at shifts 4st and 4st+2 of the word
        // (elements lo, lo+8 with lo = 3,2 | 1,0 | 7,6 | 5,4)
#pragma unroll
        for (int st = 0; st < 4; ++st) {
          const int lo0 = (st & 1) ? 1 : 3, base = (st >> 1) * 4;
          qa[g * 4 + st][h2] = pack_f16x2(v[base + lo0], v[base + lo0 + 8]);
          qa[g * 4 + st][2 + h2] = pack_f16x2(v[base + lo0 - 1], v[base + lo0 + 7]);
        }
      } else {
#pragma unroll
        for (int wi = 0; wi < 2; ++wi) {
          const int sA = g * 4 + 2 * wi;
          const float* e = &v[8 * wi];
          qa[sA][h2] = pack_f16x2(e[0], e[4]);
          qa[sA][2 + h2] = pack_f16x2(e[1], e[5]);
          qa[sA + 1][h2] = pack_f16x2(e[2], e[6]);
          qa[sA + 1][2 + h2] = pack_f16x2(e[3], e[7]);
        }
      }
    }
  }

  float oacc[NTD][4];
#pragma unroll
  for (int j = 0; j < NTD; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) oacc[j][i] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};

  // K for tokens r and 8+r, V for tokens 2c,2c+1,8+2c,9+2c of one sub-tile
  struct Tile {
    uint32_t kw[2][DG][KW];
    float ksc[2][2][DG];
    uint32_t vw[4][DG][VW];
    float vsc[4][DG];
  };
  auto load_tile = [&](int sub, Tile& T) {
    const int t0 = sub * 16;
    const int page = p.block_table[int64_t(b) * p.max_pages + t0 / p.PS];
    // row of token t0; token t0+i is at rowbase + i*slot_stride
    const int64_t rowbase = int64_t(page) * p.Hkv * p.PS + hkv * p.head_stride + (t0 % p.PS) * p.slot_stride;
    const int64_t ss = p.slot_stride;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const uint8_t* krow = p.kp + (rowbase + (nt * 8 + r) * ss) * RB;
#pragma unroll
      for (int g = 0; g < DG; ++g) {
        if constexpr (BITS == 8) {
          const uint4 q = *reinterpret_cast<const uint4*>(krow + 64 * g + 16 * c);
          T.kw[nt][g][0] = q.x;
          T.kw[nt][g][1] = q.y;
          T.kw[nt][g][2] = q.z;
          T.kw[nt][g][3] = q.w;
        } else if constexpr (BITS == 2) {
          T.kw[nt][g][0] = *reinterpret_cast<const uint32_t*>(krow + 16 * g + 4 * c);
        } else {
          const uint2 q = *reinterpret_cast<const uint2*>(krow + 32 * g + 8 * c);
          T.kw[nt][g][0] = q.x;
          T.kw[nt][g][1] = q.y;
        }
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tok = nt * 8 + 2 * c + e;
        const bool tv = t0 + tok < len;
#pragma unroll
        for (int g = 0; g < DG; ++g) T.ksc[nt][e][g] = tv ? p.ks[(rowbase + tok * ss) * DG + g] : 0.f;
      }
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int tok = (t >> 1) * 8 + 2 * c + (t & 1);
      const bool tv = t0 + tok < len;
      const uint8_t* vrow = p.vp + (rowbase + tok * ss) * RB;
#pragma unroll
      for (int g = 0; g < DG; ++g) {
        if constexpr (BITS == 8) {
          const uint2 q = *reinterpret_cast<const uint2*>(vrow + 64 * g + 8 * r);
          T.vw[t][g][0] = q.x;
          T.vw[t][g][1] = q.y;
        } else if constexpr (BITS == 2) {
          T.vw[t][g][0] = *reinterpret_cast<const uint16_t*>(vrow + 16 * g + 2 * r);
        } else {
          T.vw[t][g][0] = *reinterpret_cast<const uint32_t*>(vrow + 32 * g + 4 * r);
        }
        T.vsc[t][g] = tv ? p.vs[(rowbase + tok * ss) * DG + g] : 0.f;
      }
    }
  };

  // S = Q.K^T, online softmax and O += P.V for one 16-token sub-tile
  auto process = [&](const Tile& cur, int t0) {
    const auto& kw = cur.kw;
    const auto& ksc = cur.ksc;
    const auto& vw = cur.vw;
    const auto& vsc = cur.vsc;

    // ---- S = Q.K^T -------------------------------------------------------
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float sacc[DG][4];
#pragma unroll
      for (int g = 0; g < DG; ++g) {
#pragma unroll
        for (int i = 0; i < 4; ++i) sacc[g][i] = 0.f;
        if constexpr (BITS == 8) {
#pragma unroll
          for (int st = 0; st < 4; ++st) {
            const uint32_t w = kw[nt][g][st];
            const uint32_t bf[2] = {prmt(w, 0x64646464u, 0x4140u), prmt(w, 0x64646464u, 0x4342u)};
            mma_f16_16816(sacc[g], qa[g * 4 + st], bf);
          }
        } else if constexpr (BITS == 2) {
          const uint32_t w = kw[nt][g][0];
#pragma unroll
          for (int st = 0; st < 4; ++st) {
            const uint32_t bf[2] = {and_or(w >> (4 * st), 0x00030003u, 0x64006400u),
                                    and_or(w >> (4 * st + 2), 0x00030003u, 0x64006400u)};
            mma_f16_16816(sacc[g], qa[g * 4 + st], bf);
          }
        } else {
#pragma unroll
          for (int wi = 0; wi < 2; ++wi) {
            const uint32_t w = kw[nt][g][wi];
            const uint32_t e15 = and_or(w, 0x000F000Fu, 0x64006400u);
            const uint32_t e04 = and_or(w >> 4, 0x000F000Fu, 0x64006400u);
            const uint32_t e37 = and_or(w >> 8, 0x000F000Fu, 0x64006400u);
            const uint32_t e26 = and_or(w >> 12, 0x000F000Fu, 0x64006400u);
            const uint32_t bA[2] = {e04, e15};
            const uint32_t bB[2] = {e26, e37};
            mma_f16_16816(sacc[g], qa[g * 4 + 2 * wi], bA);
            mma_f16_16816(sacc[g], qa[g * 4 + 2 * wi + 1], bB);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = i >> 1, e = i & 1;
        float v = 0.f;
#pragma unroll
        for (int g = 0; g < DG; ++g) v += ksc[nt][e][g] * (sacc[g][i] - KOFF * qg[row][g]);
        const int tok = nt * 8 + 2 * c + e;
        s[nt][i] = (t0 + tok < len) ? v : -INFINITY;
      }
    }

    // ---- online softmax (rows r and r+8) --------------------------------
    float pr[2][4];
#pragma unroll
    for (int row = 0; row < 2; ++row) {
      float mt = fmaxf(fmaxf(s[0][2 * row], s[0][2 * row + 1]), fmaxf(s[1][2 * row], s[1][2 * row + 1]));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      const float mnew = fmaxf(m_run[row], mt);
      const bool none = (mnew == -INFINITY);
      const float alpha = none ? 1.f : exp2f(m_run[row] - mnew);
      float lsum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pv = none ? 0.f : exp2f(s[nt][2 * row + e] - mnew);
          pr[nt][2 * row + e] = pv;
          lsum += pv;
        }
      l_run[row] = l_run[row] * alpha + lsum;
      m_run[row] = mnew;
#pragma unroll
      for (int j = 0; j < NTD; ++j) {
        oacc[j][2 * row] *= alpha;
        oacc[j][2 * row + 1] *= alpha;
      }
    }

    // ---- O += P.V --------------------------------------------------------
    const uint32_t pa[4] = {pack_f16x2(pr[0][0], pr[0][1]), pack_f16x2(pr[0][2], pr[0][3]),
                            pack_f16x2(pr[1][0], pr[1][1]), pack_f16x2(pr[1][2], pr[1][3])};
    uint32_t vs01[DG], vs23[DG];
#pragma unroll
    for (int g = 0; g < DG; ++g) {
      vs01[g] = pack_f16x2(vsc[0][g], vsc[1][g]);
      vs23[g] = pack_f16x2(vsc[2][g], vsc[3][g]);
    }
    const uint32_t off2 = pack_f16x2(KOFF, KOFF);
#pragma unroll
    for (int j = 0; j < NTD; ++j) {
      const int gj = j >> 3, jj = j & 7;
      uint32_t x01, x23;
      if constexpr (BITS == 8) {
        const int wsel = jj >> 2, k = jj & 3;
        const uint32_t sel = uint32_t(k | (k << 4) | ((4 + k) << 8) | ((4 + k) << 12));
        x01 = and_or(prmt(vw[0][gj][wsel], vw[1][gj][wsel], sel), 0x00FF00FFu, 0x64006400u);
        x23 = and_or(prmt(vw[2][gj][wsel], vw[3][gj][wsel], sel), 0x00FF00FFu, 0x64006400u);
      } else if constexpr (BITS == 2) {
        // element 8r+jj: byte jj/4 of the two loaded, crumb jj%4 (most significant first)
        const int k = jj >> 2, sh = 6 - 2 * (jj & 3);
        const uint32_t sel = uint32_t(k | (k << 4) | ((4 + k) << 8) | ((4 + k) << 12));
        x01 = and_or(prmt(vw[0][gj][0], vw[1][gj][0], sel) >> sh, 0x00030003u, 0x64006400u);
        x23 = and_or(prmt(vw[2][gj][0], vw[3][gj][0], sel) >> sh, 0x00030003u, 0x64006400u);
      } else {
        const int k = jj >> 1;
        const uint32_t sel = uint32_t(k | (k << 4) | ((4 + k) << 8) | ((4 + k) << 12));
        uint32_t y01 = prmt(vw[0][gj][0], vw[1][gj][0], sel);
        uint32_t y23 = prmt(vw[2][gj][0], vw[3][gj][0], sel);
        if ((jj & 1) == 0) {
          y01 >>= 4;
          y23 >>= 4;
        }
        x01 = and_or(y01, 0x000F000Fu, 0x64006400u);
        x23 = and_or(y23, 0x000F000Fu, 0x64006400u);
      }
      const uint32_t bfr[2] = {hmul2_u(hsub2_u(x01, off2), vs01[gj]), hmul2_u(hsub2_u(x23, off2), vs23[gj])};
      mma_f16_16816(oacc[j], pa, bfr);
    }
  };

  extern __shared__ __align__(1024) uint8_t attn_smem[];
  bool aborted = false;
  if constexpr (!RING) {
    Tile nxt;
    if (sub_begin + warp < sub_end) load_tile(sub_begin + warp, nxt);
    for (int sub = sub_begin + warp; sub < sub_end; sub += 4) {
      const Tile cur = nxt;  // this sub-tile; the next one is loaded while it is computed
      if (sub + 4 < sub_end) load_tile(sub + 4, nxt);
      process(cur, sub * 16);
    }
  } else {
    // ---- page ring: warp 4 streams whole pages (TMA tiles of K/V codes, bulk
    // copies of their scales) into ATTN_RING slots; warps 0-3 compute from them
    uint64_t* full = reinterpret_cast<uint64_t*>(attn_smem + p.ring_bytes - 128);
    uint64_t* empty = full + ATTN_RING;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + ATTN_RING);
    if (threadIdx.x == 0) {
      for (int i = 0; i < ATTN_RING; ++i) {
        mbar_init(&full[i], 1);
        mbar_init(&empty[i], 4);
      }
      *abort_flag = 0;
      fence_mbarrier_init();
    }
    __syncthreads();
    const int spp = p.PS / 16;
    const int pg0 = sub_begin / spp;
    const int npg = sub_end > sub_begin ? (sub_end + spp - 1) / spp - pg0 : 0;
    constexpr int RB_ = D * BITS / 8;
    const int code_bytes = p.PS * RB_, sc_bytes = p.PS * DG * 4;
    if (warp == 4) {
      if (lane == 0 && !producers_stalled()) {  // test control: stalled producers issue nothing
        int jj = 0;
        for (; jj < npg; ++jj) {
          const int slot = jj % ATTN_RING;
          if (jj >= ATTN_RING && !mbar_wait_bounded(&empty[slot], uint32_t(((jj / ATTN_RING) - 1) & 1))) {
            *abort_flag = 1;
            break;
          }
          if (*abort_flag) break;
          const int page = p.block_table[int64_t(b) * p.max_pages + pg0 + jj];
          const int64_t rowbase = (int64_t(page) * p.Hkv + hkv) * p.PS;
          uint8_t* sb = attn_smem + slot * p.slot_bytes;
          mbar_arrive_expect_tx(&full[slot], uint32_t(2 * code_bytes + 2 * sc_bytes));
          tma_load_2d(sb, &tmk, 0, int(rowbase), &full[slot]);
          tma_load_2d(sb + code_bytes, &tmv, 0, int(rowbase), &full[slot]);
          bulk_g2s(sb + 2 * code_bytes, p.ks + rowbase * DG, uint32_t(sc_bytes), &full[slot]);
          bulk_g2s(sb + 2 * code_bytes + sc_bytes, p.vs + rowbase * DG, uint32_t(sc_bytes), &full[slot]);
        }
        // copies already issued land before the CTA goes away
        for (int k = 1; k <= ATTN_RING && jj - k >= 0; ++k)
          mbar_wait_bounded(&full[(jj - k) % ATTN_RING], uint32_t(((jj - k) / ATTN_RING) & 1), 100000000ull);
      }
      __syncwarp();
    } else {
      for (int jj = 0; jj < npg; ++jj) {
        const int slot = jj % ATTN_RING;
        const bool ok = !*abort_flag && mbar_wait_bounded(&full[slot], uint32_t((jj / ATTN_RING) & 1));
        if (!__all_sync(0xffffffffu, ok)) {
          if (lane == 0) *abort_flag = 1;
          aborted = true;
          break;
        }
        const uint8_t* kb = attn_smem + slot * p.slot_bytes;
        const uint8_t* vb = kb + code_bytes;
        const float* ksb = reinterpret_cast<const float*>(kb + 2 * code_bytes);
        const float* vsb = ksb + p.PS * DG;
        const int s_lo = max(sub_begin, (pg0 + jj) * spp), s_hi = min(sub_end, (pg0 + jj + 1) * spp);
        for (int sub = s_lo; sub < s_hi; ++sub) {
          if (((sub - sub_begin) & 3) != warp) continue;
          const int t0 = sub * 16;
          const int lr = t0 % p.PS;  // first row of the sub-tile in the page
          Tile T;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int row = lr + nt * 8 + r;
#pragma unroll
            for (int g = 0; g < DG; ++g) {
              if constexpr (BITS == 8) {
                const uint4 q = *reinterpret_cast<const uint4*>(kb + swz_off<RB_>(row, 64 * g + 16 * c));
                T.kw[nt][g][0] = q.x;
                T.kw[nt][g][1] = q.y;
                T.kw[nt][g][2] = q.z;
                T.kw[nt][g][3] = q.w;
              } else if constexpr (BITS == 2) {
                T.kw[nt][g][0] = *reinterpret_cast<const uint32_t*>(kb + swz_off<RB_>(row, 16 * g + 4 * c));
              } else {
                const uint2 q = *reinterpret_cast<const uint2*>(kb + swz_off<RB_>(row, 32 * g + 8 * c));
                T.kw[nt][g][0] = q.x;
                T.kw[nt][g][1] = q.y;
              }
            }
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int tok = nt * 8 + 2 * c + e;
              const bool tv = t0 + tok < len;
#pragma unroll
              for (int g = 0; g < DG; ++g) T.ksc[nt][e][g] = tv ? ksb[(lr + tok) * DG + g] : 0.f;
            }
          }
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int tok = (t >> 1) * 8 + 2 * c + (t & 1);
            const bool tv = t0 + tok < len;
#pragma unroll
            for (int g = 0; g < DG; ++g) {
              if constexpr (BITS == 8) {
                const uint2 q = *reinterpret_cast<const uint2*>(vb + swz_off<RB_>(lr + tok, 64 * g + 8 * r));
                T.vw[t][g][0] = q.x;
                T.vw[t][g][1] = q.y;
              } else if constexpr (BITS == 2) {
                T.vw[t][g][0] = *reinterpret_cast<const uint16_t*>(vb + swz_off<RB_>(lr + tok, 16 * g + 2 * r));
              } else {
                T.vw[t][g][0] = *reinterpret_cast<const uint32_t*>(vb + swz_off<RB_>(lr + tok, 32 * g + 4 * r));
              }
              T.vsc[t][g] = tv ? vsb[(lr + tok) * DG + g] : 0.f;
            }
          }
          process(T, t0);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
    }
  }

  // ---- merge the 4 warps through shared memory -----------------------------
  float* sm = reinterpret_cast<float*>(attn_smem + (RING ? p.ring_bytes : 0));
  float* sm_o = sm;                      // [4][G][D]
  float* sm_ml = sm + 4 * G * D;         // [4][G][2]
#pragma unroll
  for (int row = 0; row < 2; ++row) {
    float l = l_run[row];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int head = r + 8 * row;
    if (head < G && warp < 4) {
      if (c == 0) {
        sm_ml[(warp * G + head) * 2 + 0] = m_run[row];
        sm_ml[(warp * G + head) * 2 + 1] = l;
      }
#pragma unroll
      for (int j = 0; j < NTD; ++j) {
        const int gj = j >> 3, jj = j & 7;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int d = 64 * gj + 8 * (2 * c + e) + jj;
          sm_o[(warp * G + head) * D + d] = oacc[j][2 * row + e];
        }
      }
    }
  }
  __syncthreads();
  if (aborted && (threadIdx.x & 31) == 0) report_timeout(nullptr);  // a page wait gave up
  const int hq0 = hkv * G;
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int head = idx / D, d = idx % D;
    float mstar = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mstar = fmaxf(mstar, sm_ml[(w * G + head) * 2]);
    float o = 0.f, l = 0.f;
    if (mstar != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(sm_ml[(w * G + head) * 2] - mstar);
        o += f * sm_o[(w * G + head) * D + d];
        l += f * sm_ml[(w * G + head) * 2 + 1];
      }
    }
    const int64_t bh = int64_t(b) * p.Hq + hq0 + head;
    if (p.n_splits == 1) {
      p.out[bh * D + d] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
    } else {
      p.o_part[(bh * p.n_splits + split) * D + d] = o;
      if (d == 0) {
        p.ml_part[(bh * p.n_splits + split) * 2 + 0] = mstar;
        p.ml_part[(bh * p.n_splits + split) * 2 + 1] = l;
      }
    }
  }
}

// 8x8 transpose of 16-bit elements across the warp: lane (r, c) holds
// elements (r, 2c), (r, 2c+1) before and (2c, r), (2c+1, r) after.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(x));
  return d;
}

// ---------------------------------------------------------------------------
// Token-row form for 8-bit codes, D = 128, G <= 8, head-major pages (the
// decode shape of the grouped-query models here).  The MMA's M side is 16
// tokens and its N side the G query heads of the KV head, so with G = 8 no
// MMA row is padding (the form above fills 8 of its 16 rows):
//   S^T = K.Q^T    A = K codes as fp16 1024+code (one prmt per two codes),
//                  B = q^T (fp16, pre-scaled by softmax_scale*log2(e));
//                  per 64-wide group s = kscale*(acc - (1024+127)*sum(q))
//   online softmax per head over the 8 lanes sharing its column
//   P' = P*vscale  per token and group, moved into the B layout of the next
//                  MMA with one 8x8 transpose per 8 tokens
//   O^T += V^T.P'^T  A = V codes as fp16 1024+code (two tokens per register),
//                  plus one MMA of an all-ones A per group that accumulates
//                  sum(P'); O = acc - (1024+127)*sum(P') at the end.
// Inside each 8-token half, MMA row i is page row sigma(i) (sigma = 0 6 1 7
// 4 2 5 3): with the 128B swizzle of the page tiles that makes every K and V
// fragment read of a warp hit 32 distinct banks.  The page ring and the
// split partials are those of the kernel above; the producer warp leaves once
// its copies have landed, and the 4 compute warps merge through shared memory
// behind a named barrier of their own.
// ex2.approx.ftz: 2^x (-inf gives +0), the softmax exponential in base 2
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// NT = 16-token tiles a warp takes per step (2 when the pages hold an even
// number of tiles): the tiles' MMA chains, loads and conversions interleave,
// and the softmax max and the O rescale are paid once per NT tiles.
template <int D, int NT>
__global__ void __launch_bounds__(160, 2) qkv_decode_attn_t8_kernel(const AttnParams p,
                                                                    const __grid_constant__ CUtensorMap tmk,
                                                                    const __grid_constant__ CUtensorMap tmv) {
  pdl_enter();
  static_assert(D == 128, "token-row form: 128-byte code rows");
  constexpr int DG = D / 64;  // quantization groups per row
  constexpr int RB = D;       // bytes per 8-bit code row
  constexpr float KOFF = 1024.f + 127.f;
  constexpr uint32_t SIGMA = 0x35247160u;  // nibble i = page row of MMA row i (mod 8)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int G = p.G;

  const int sg = (SIGMA >> (4 * g)) & 7;       // page row of MMA rows g (and 8+sg of g+8)
  const int sv0 = (SIGMA >> (8 * c)) & 7;      // page row of token 2c (B side of P.V)
  const int sv1 = (SIGMA >> (8 * c + 4)) & 7;  // page row of token 2c+1
  // byte offsets inside a swizzled code row: K (16 bytes, dims 64grp+16c..)
  // for rows sg / 8+sg; V (8 bytes, dims 64grp+vdim(g)..) for rows sv0 / sv1
  const int vdim = 32 * ((g >> 1) & 1) + 16 * (g >> 2) + 8 * (g & 1);
  int kcol[DG], vcol0[DG], vcol1[DG];
#pragma unroll
  for (int grp = 0; grp < DG; ++grp) {
    kcol[grp] = sg * RB + ((((4 * grp) | c) ^ sg) << 4);
    const int ch = (64 * grp + vdim) >> 4;
    vcol0[grp] = sv0 * RB + ((ch ^ sv0) << 4) + 8 * (g & 1);
    vcol1[grp] = sv1 * RB + ((ch ^ sv1) << 4) + 8 * (g & 1);
  }

  extern __shared__ __align__(1024) uint8_t attn_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(attn_smem + p.ring_bytes - 128);
  uint64_t* empty = full + ATTN_RING;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + ATTN_RING);
  float* sm = reinterpret_cast<float*>(attn_smem + p.ring_bytes);
  float* sm_o = sm;               // [4][G][D]
  float* sm_ml = sm + 4 * G * D;  // [4][G][2]
  if (threadIdx.x == 0) {
    for (int i = 0; i < ATTN_RING; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  // the CTA's pages: pair (blockIdx.z, blockIdx.y), context split blockIdx.x
  const int b = blockIdx.z, hkv = blockIdx.y;
  const int len = p.seq_lens[b];
  const int n_sub = (len + 15) / 16;
  const int per_split = (n_sub + p.n_splits - 1) / p.n_splits;
  const int sub_begin = int(blockIdx.x) * per_split;
  const int sub_end = min(n_sub, sub_begin + per_split);

  const int spp = p.PS / 16;
  const int pg0 = sub_begin / spp;
  const int npg = sub_end > sub_begin ? (sub_end + spp - 1) / spp - pg0 : 0;
  const int code_bytes = p.PS * RB, sc_bytes = p.PS * DG * 4;
  if (warp == 4) {
    if (lane == 0 && !producers_stalled()) {  // test control: stalled producers issue nothing
      int it = 0;  // pages issued (ring position)
      for (; it < npg; ++it) {
        const int slot = it % ATTN_RING;
        if (it >= ATTN_RING && !mbar_wait_bounded_backoff(&empty[slot], uint32_t(((it / ATTN_RING) - 1) & 1))) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const int page = p.block_table[int64_t(b) * p.max_pages + pg0 + it];
        const int64_t rowbase = (int64_t(page) * p.Hkv + hkv) * p.PS;
        uint8_t* sb = attn_smem + slot * p.slot_bytes;
        mbar_arrive_expect_tx(&full[slot], uint32_t(2 * code_bytes + 2 * sc_bytes));
        tma_load_2d(sb, &tmk, 0, int(rowbase), &full[slot]);
        tma_load_2d(sb + code_bytes, &tmv, 0, int(rowbase), &full[slot]);
        bulk_g2s(sb + 2 * code_bytes, p.ks + rowbase * DG, uint32_t(sc_bytes), &full[slot]);
        bulk_g2s(sb + 2 * code_bytes + sc_bytes, p.vs + rowbase * DG, uint32_t(sc_bytes), &full[slot]);
      }
      // copies already issued land before the CTA goes away
      for (int k = 1; k <= ATTN_RING && it - k >= 0; ++k)
        mbar_wait_bounded(&full[(it - k) % ATTN_RING], uint32_t(((it - k) / ATTN_RING) & 1), 100000000ull);
    }
    __syncwarp();
    return;
  }

  // ---- consumer warps 0..3 ---------------------------------------------------
  const uint32_t ONE2 = 0x3C003C00u;
  const uint32_t ones[4] = {ONE2, ONE2, ONE2, ONE2};
  {
    uint32_t qb[DG * 4][2];
    float kq[2][DG];  // heads 2c, 2c+1
    // ---- q^T fragments (head g, dims 64grp+16c+[0,16)) and (1024+127)*sum(q)
    {
      const bool hv = g < G;
      const __nv_bfloat16* qrow = p.q + (int64_t(b) * p.Hq + int64_t(hkv) * G + g) * D;
#pragma unroll
      for (int grp = 0; grp < DG; ++grp) {
        float v[16];
        if (hv) {
          const uint4* src = reinterpret_cast<const uint4*>(qrow + 64 * grp + 16 * c);
          const uint4 a = src[0], bb = src[1];
          const uint32_t w[8] = {a.x, a.y, a.z, a.w, bb.x, bb.y, bb.z, bb.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
            v[2 * i] = round_f16(__low2float(h) * p.qscale);
            v[2 * i + 1] = round_f16(__high2float(h) * p.qscale);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.f;
        }
        float part = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) part += v[i];
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
#pragma unroll
        for (int st = 0; st < 4; ++st) {
          qb[grp * 4 + st][0] = pack_f16x2(v[4 * st], v[4 * st + 1]);
          qb[grp * 4 + st][1] = pack_f16x2(v[4 * st + 2], v[4 * st + 3]);
        }
        kq[0][grp] = KOFF * __shfl_sync(0xffffffffu, part, 8 * c);
        kq[1][grp] = KOFF * __shfl_sync(0xffffffffu, part, 8 * c + 4);
      }
    }

    float oacc[DG * 4][4];
    float oone[DG][4];
#pragma unroll
    for (int j = 0; j < DG * 4; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) oacc[j][i] = 0.f;
#pragma unroll
    for (int j = 0; j < DG; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) oone[j][i] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_run[2] = {0.f, 0.f};  // this lane's rows only; summed over the 8 row lanes at the end
    for (int it = 0; it < npg; ++it) {
      const int slot = it % ATTN_RING;
      const bool ok = !*abort_flag && mbar_wait_bounded(&full[slot], uint32_t((it / ATTN_RING) & 1));
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      const uint8_t* kb = attn_smem + slot * p.slot_bytes;
      const uint8_t* vb = kb + code_bytes;
      const float* ksb = reinterpret_cast<const float*>(kb + 2 * code_bytes);
      const float* vsb = ksb + p.PS * DG;
      const int s_lo = max(sub_begin, (pg0 + it) * spp), s_hi = min(sub_end, (pg0 + it + 1) * spp);
      const int nstep = (s_hi - s_lo + NT - 1) / NT;
      for (int k = 0; k < nstep; ++k) {
        if (((it * (spp / NT) + k) & 3) != warp) continue;
        const int sub0 = s_lo + NT * k;
            uint4 kw[NT][2][DG];
            uint2 vw[NT][4][DG];  // tokens 2c, 2c+1, 2c+8, 2c+9
            bool valid[NT][2];
            float ksc[NT][2][DG], vsc[NT][2][DG];
    #pragma unroll
            for (int t = 0; t < NT; ++t) {
              const bool here = sub0 + t < s_hi;  // warp-uniform
              const int t0 = (sub0 + t) * 16;
              const int lr = here ? t0 % p.PS : 0;  // first page row of the tile (a multiple of 16)
              const uint8_t* kt = kb + lr * RB;
              const uint8_t* vt = vb + lr * RB;
    #pragma unroll
              for (int grp = 0; grp < DG; ++grp) {
                kw[t][0][grp] = *reinterpret_cast<const uint4*>(kt + kcol[grp]);
                kw[t][1][grp] = *reinterpret_cast<const uint4*>(kt + 8 * RB + kcol[grp]);
                vw[t][0][grp] = *reinterpret_cast<const uint2*>(vt + vcol0[grp]);
                vw[t][1][grp] = *reinterpret_cast<const uint2*>(vt + vcol1[grp]);
                vw[t][2][grp] = *reinterpret_cast<const uint2*>(vt + 8 * RB + vcol0[grp]);
                vw[t][3][grp] = *reinterpret_cast<const uint2*>(vt + 8 * RB + vcol1[grp]);
              }
    #pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int row = lr + 8 * h + sg;
                valid[t][h] = here && t0 + 8 * h + sg < len;
                const float2 kk = *reinterpret_cast<const float2*>(ksb + row * DG);
                const float2 vv = *reinterpret_cast<const float2*>(vsb + row * DG);
                ksc[t][h][0] = kk.x;
                ksc[t][h][1] = kk.y;
                vsc[t][h][0] = valid[t][h] ? vv.x : 0.f;
                vsc[t][h][1] = valid[t][h] ? vv.y : 0.f;
              }
            }

            // ---- S^T = K.Q^T ---------------------------------------------------
            float s[NT][4];
    #pragma unroll
            for (int t = 0; t < NT; ++t) {
              float sacc[DG][4];
    #pragma unroll
              for (int grp = 0; grp < DG; ++grp) {
    #pragma unroll
                for (int i = 0; i < 4; ++i) sacc[grp][i] = 0.f;
                const uint32_t k0[4] = {kw[t][0][grp].x, kw[t][0][grp].y, kw[t][0][grp].z, kw[t][0][grp].w};
                const uint32_t k1[4] = {kw[t][1][grp].x, kw[t][1][grp].y, kw[t][1][grp].z, kw[t][1][grp].w};
    #pragma unroll
                for (int st = 0; st < 4; ++st) {
                  const uint32_t a[4] = {prmt(k0[st], 0x64646464u, 0x4140u), prmt(k1[st], 0x64646464u, 0x4140u),
                                         prmt(k0[st], 0x64646464u, 0x4342u), prmt(k1[st], 0x64646464u, 0x4342u)};
                  mma_f16_16816(sacc[grp], a, qb[grp * 4 + st]);
                }
              }
    #pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int h = i >> 1, e = i & 1;
                float v = 0.f;
    #pragma unroll
                for (int grp = 0; grp < DG; ++grp) v += ksc[t][h][grp] * (sacc[grp][i] - kq[e][grp]);
                s[t][i] = valid[t][h] ? v : -INFINITY;
              }
            }

            // ---- online softmax (heads 2c, 2c+1 over the 8 lanes of a column) --
            float pr[NT][4];
    #pragma unroll
            for (int e = 0; e < 2; ++e) {
              float mt = fmaxf(s[0][e], s[0][2 + e]);
    #pragma unroll
              for (int t = 1; t < NT; ++t) mt = fmaxf(mt, fmaxf(s[t][e], s[t][2 + e]));
              mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
              mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
              mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
              const float mnew = fmaxf(m_run[e], mt);
              const bool none = (mnew == -INFINITY);
              const float alpha = none ? 1.f : fast_exp2(m_run[e] - mnew);
              float lsum = 0.f;
    #pragma unroll
              for (int t = 0; t < NT; ++t) {
                pr[t][e] = none ? 0.f : fast_exp2(s[t][e] - mnew);
                pr[t][2 + e] = none ? 0.f : fast_exp2(s[t][2 + e] - mnew);
                lsum += pr[t][e] + pr[t][2 + e];
              }
              l_run[e] = l_run[e] * alpha + lsum;
              m_run[e] = mnew;
    #pragma unroll
              for (int j = 0; j < DG * 4; ++j) {
                oacc[j][e] *= alpha;
                oacc[j][2 + e] *= alpha;
              }
    #pragma unroll
              for (int j = 0; j < DG; ++j) {
                oone[j][e] *= alpha;
                oone[j][2 + e] *= alpha;
              }
            }

            // ---- O^T += V^T.P'^T ------------------------------------------------
    #pragma unroll
            for (int t = 0; t < NT; ++t) {
    #pragma unroll
              for (int grp = 0; grp < DG; ++grp) {
                const uint32_t xlo = pack_f16x2(pr[t][0] * vsc[t][0][grp], pr[t][1] * vsc[t][0][grp]);
                const uint32_t xhi = pack_f16x2(pr[t][2] * vsc[t][1][grp], pr[t][3] * vsc[t][1][grp]);
                const uint32_t bp[2] = {movmatrix_trans(xlo), movmatrix_trans(xhi)};
                mma_f16_16816(oone[grp], ones, bp);
    #pragma unroll
                for (int jl = 0; jl < 4; ++jl) {
                  const int bs = 2 * (jl & 1);
                  const uint32_t sel_lo = uint32_t(bs | (bs << 4) | ((4 + bs) << 8) | ((4 + bs) << 12));
                  const uint32_t sel_hi = sel_lo + 0x1111u;
                  const uint32_t w0 = (jl >> 1) ? vw[t][0][grp].y : vw[t][0][grp].x;
                  const uint32_t w1 = (jl >> 1) ? vw[t][1][grp].y : vw[t][1][grp].x;
                  const uint32_t w2 = (jl >> 1) ? vw[t][2][grp].y : vw[t][2][grp].x;
                  const uint32_t w3 = (jl >> 1) ? vw[t][3][grp].y : vw[t][3][grp].x;
                  const uint32_t a[4] = {and_or(prmt(w0, w1, sel_lo), 0x00FF00FFu, 0x64006400u),
                                         and_or(prmt(w0, w1, sel_hi), 0x00FF00FFu, 0x64006400u),
                                         and_or(prmt(w2, w3, sel_lo), 0x00FF00FFu, 0x64006400u),
                                         and_or(prmt(w2, w3, sel_hi), 0x00FF00FFu, 0x64006400u)};
                  mma_f16_16816(oacc[grp * 4 + jl], a, bp);
                }
              }
            }
          }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }

    // ---- merge the 4 warps through shared memory (the producer warp has left)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float l = l_run[e];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      const int head = 2 * c + e;
      if (head < G) {
        if (g == 0) {
          sm_ml[(warp * G + head) * 2 + 0] = m_run[e];
          sm_ml[(warp * G + head) * 2 + 1] = l;
        }
#pragma unroll
        for (int j = 0; j < DG * 4; ++j) {
          const int grp = j >> 2, jl = j & 3;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int d = 64 * grp + vdim + 2 * jl + h;
            sm_o[(warp * G + head) * D + d] = oacc[j][2 * h + e] - KOFF * oone[grp][2 * h + e];
          }
        }
      }
    }
    named_bar_sync(1, 128);
    if (threadIdx.x == 0 && *abort_flag) report_timeout(nullptr);  // a page wait gave up
    const int hq0 = hkv * G;
    for (int idx = threadIdx.x; idx < G * D; idx += 128) {
      const int head = idx / D, d = idx % D;
      float mstar = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) mstar = fmaxf(mstar, sm_ml[(w * G + head) * 2]);
      float o = 0.f, l = 0.f;
      if (mstar != -INFINITY) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float f = exp2f(sm_ml[(w * G + head) * 2] - mstar);
          o += f * sm_o[(w * G + head) * D + d];
          l += f * sm_ml[(w * G + head) * 2 + 1];
        }
      }
      const int64_t bh = int64_t(b) * p.Hq + hq0 + head;
      if (p.n_splits == 1) {
        p.out[bh * D + d] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
      } else {
        const int split = blockIdx.x;
        p.o_part[(bh * p.n_splits + split) * D + d] = o;
        if (d == 0) {
          p.ml_part[(bh * p.n_splits + split) * 2 + 0] = mstar;
          p.ml_part[(bh * p.n_splits + split) * 2 + 1] = l;
        }
      }
    }
  }
}

__global__ void attn_combine_kernel(const float* __restrict__ o_part, const float* __restrict__ ml_part,
                                    int n_splits, int D, __nv_bfloat16* __restrict__ out) {
  pdl_enter();
  const int64_t bh = blockIdx.x;
  const float* ml = ml_part + bh * n_splits * 2;
  float mstar = -INFINITY;
  for (int s = 0; s < n_splits; ++s) mstar = fmaxf(mstar, ml[2 * s]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f, l = 0.f;
    if (mstar != -INFINITY) {
      for (int s = 0; s < n_splits; ++s) {
        const float f = exp2f(ml[2 * s] - mstar);
        o += f * o_part[(bh * n_splits + s) * D + d];
        l += f * ml[2 * s + 1];
      }
    }
    out[bh * D + d] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
  }
}

// K or V code pages as a 2-D uint8 tensor of rows of RB bytes (one row per
// token and KV head); box = one page of one head (page_size rows), swizzled
// so the warps' fragment reads hit distinct banks.  The row count is not
// known here; only rows named by the block table are ever addressed.
static int make_kv_map(CUtensorMap* map, const uint8_t* base, int RB, int PS) {
  const cuuint64_t dims[2] = {cuuint64_t(RB), cuuint64_t(1) << 31};
  const cuuint64_t strides[1] = {cuuint64_t(RB)};
  const cuuint32_t box[2] = {cuuint32_t(RB), cuuint32_t(PS)};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = RB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : RB == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                           : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B2F_OK : B2F_ERR_INVALID;
}

template <int BITS, int D>
static int launch_attn(AttnParams p, cudaStream_t st) {
  constexpr int RB = D * BITS / 8;
  constexpr int DG = D / 64;
  const int merge = (4 * p.G * D + 4 * p.G * 2) * int(sizeof(float));
  // page ring: head-major pages whose code rows fit one swizzled TMA box row
  constexpr bool RING_OK = D <= 128 && RB <= 128 && RB % 32 == 0;  // D = 256 would spill registers
  // (and whose ATTN_RING pages fit the 227 KB of shared memory of one CTA;
  // larger pages take the direct-load form)
  const int slot_bytes = (2 * p.PS * RB + 2 * p.PS * DG * 4 + 1023) / 1024 * 1024;
  const bool ring = RING_OK && p.head_stride == p.PS && p.slot_stride == 1 && p.PS <= 256 &&
                    ATTN_RING * slot_bytes + 128 + merge <= 227 * 1024 && aligned(p.ks, 16) &&
                    aligned(p.vs, 16) && get_encoder() == B2F_OK;
  CUtensorMap mk{}, mv{};
  int smem = merge;
  if (ring) {
    if (make_kv_map(&mk, p.kp, RB, p.PS) != B2F_OK || make_kv_map(&mv, p.vp, RB, p.PS) != B2F_OK)
      return B2F_ERR_INVALID;
    p.slot_bytes = slot_bytes;
    p.ring_bytes = ATTN_RING * p.slot_bytes + 128;
    smem = p.ring_bytes + merge;
  }
  auto kern = qkv_decode_attn_kernel<BITS, D, false>;
  if constexpr (RING_OK) {
    if (ring) kern = qkv_decode_attn_kernel<BITS, D, true>;
  }
  if constexpr (BITS == 8 && D == 128) {
    if (ring && p.G <= 8) kern = (p.PS / 16) % 2 == 0 ? qkv_decode_attn_t8_kernel<D, 2> : qkv_decode_attn_t8_kernel<D, 1>;
  }
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return B2F_ERR_CUDA;
    }
  }
  const dim3 grid{unsigned(p.n_splits), unsigned(p.Hkv), unsigned(p.B)};
  int rc = launch_kernel(kern, grid, dim3{ring ? 160u : 128u}, size_t(smem), st, p, mk, mv);
  if (rc != B2F_OK || p.n_splits == 1) return rc;
  return launch_kernel(attn_combine_kernel, dim3{unsigned(int64_t(p.B) * p.Hq)}, dim3{128}, 0, st,
                       static_cast<const float*>(p.o_part), static_cast<const float*>(p.ml_part), p.n_splits, D,
                       p.out);
}

B2F_DEFINE_WAIT_CONTROLS(attn)

}  // namespace b2f

using namespace b2f;

extern "C" {

int64_t b2f_qkv_decode_attn_workspace_bytes(int64_t B, int64_t Hq, int64_t D, int n_splits) {
  if (B <= 0 || Hq <= 0 || D <= 0 || n_splits <= 1) return 0;
  return B * Hq * n_splits * (D + 2) * int64_t(sizeof(float));
}

int b2f_qkv_decode_attn(const void* q, const uint8_t* k_pages, const float* k_scales,
                        const uint8_t* v_pages, const float* v_scales, const int32_t* block_table,
                        int64_t max_pages, const int32_t* seq_lens, int64_t B, int64_t Hq,
                        int64_t Hkv, int64_t D, int64_t page_size, int64_t head_stride,
                        int64_t slot_stride, int bits, int group_size, float softmax_scale,
                        int n_splits, void* workspace, int64_t workspace_bytes, void* out,
                        void* stream) {
  if (!(bits == 2 || bits == 4 || bits == 8)) return B2F_ERR_UNSUPPORTED;
  if (!(D == 64 || D == 128 || D == 256) || group_size != 64) return B2F_ERR_UNSUPPORTED;
  if (B < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0) return B2F_ERR_INVALID;
  if (Hq / Hkv > 16) return B2F_ERR_UNSUPPORTED;
  if (page_size <= 0 || page_size % 16 != 0 || max_pages <= 0 || n_splits < 1) return B2F_ERR_INVALID;
  // the Hkv*page_size rows of a page must be covered exactly once
  const bool head_major = head_stride == page_size && slot_stride == 1;
  const bool token_major = head_stride == 1 && slot_stride == Hkv;
  if (!head_major && !token_major) return B2F_ERR_INVALID;
  if (B == 0) return B2F_OK;
  if (B > 65535 || Hkv > 65535 || n_splits > 65535) return B2F_ERR_UNSUPPORTED;
  if (!q || !k_pages || !k_scales || !v_pages || !v_scales || !block_table || !seq_lens || !out)
    return B2F_ERR_INVALID;
  if (!aligned(q, 16) || !aligned(k_pages, 16) || !aligned(v_pages, 16) || !aligned(k_scales, 4) ||
      !aligned(v_scales, 4))
    return B2F_ERR_ALIGN;
  AttnParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.kp = k_pages;
  p.ks = k_scales;
  p.vp = v_pages;
  p.vs = v_scales;
  p.block_table = block_table;
  p.max_pages = max_pages;
  p.seq_lens = seq_lens;
  p.B = int(B);
  p.Hq = int(Hq);
  p.Hkv = int(Hkv);
  p.G = int(Hq / Hkv);
  p.PS = int(page_size);
  p.head_stride = head_stride;
  p.slot_stride = slot_stride;
  p.n_splits = n_splits;
  p.qscale = softmax_scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  if (n_splits > 1) {
    const int64_t need = b2f_qkv_decode_attn_workspace_bytes(B, Hq, D, n_splits);
    if (!workspace || workspace_bytes < need) return B2F_ERR_WORKSPACE;
    if (!aligned(workspace, 16)) return B2F_ERR_ALIGN;
    p.o_part = static_cast<float*>(workspace);
    p.ml_part = p.o_part + B * Hq * n_splits * D;
  }
  cudaStream_t st = as_stream(stream);
  if (bits == 8) {
    if (D == 64) return launch_attn<8, 64>(p, st);
    if (D == 128) return launch_attn<8, 128>(p, st);
    return launch_attn<8, 256>(p, st);
  }
  if (bits == 2) {
    if (D == 64) return launch_attn<2, 64>(p, st);
    if (D == 128) return launch_attn<2, 128>(p, st);
    return launch_attn<2, 256>(p, st);
  }
  if (D == 64) return launch_attn<4, 64>(p, st);
  if (D == 128) return launch_attn<4, 128>(p, st);
  return launch_attn<4, 256>(p, st);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of b2f_qkv_decode_attn.
//
// Some callers cannot allocate device memory at the point where they run
// decode attention: a host binding (cgo / JNI / a plain C program) that has no
// device allocator of its own, a serving loop whose GPU memory is already
// fully owned by another framework's pool, or a latency-critical path where a
// cudaMalloc (which can synchronise the whole device) is not acceptable.  For
// them the split-K partial results live in the fixed device array below
// instead of a caller-provided workspace.
//
// The array is B2F_ATTN_NOALLOC_SCRATCH_BYTES (4 MiB) and is part of the
// library image: every GPU that loads the library holds it until the process
// exits.  All calls on a device share it and it keeps the previous call's
// contents; the kernels overwrite every byte they later read, so nothing has
// to be cleared between calls.  Calls that overlap on the GPU (different
// streams, or different host threads on the same device) race on it.
// ---------------------------------------------------------------------------
#include <mutex>

namespace b2f {

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[B2F_ATTN_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array for the current device.  The host-side
// symbol is only a stand-in, so the address is looked up with
// cudaGetSymbolAddress once per device (with that device current) and cached.
static int attn_noalloc_scratch(void** out) {
  constexpr int kMaxDevices = 64;
  static void* cache[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return B2F_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return B2F_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_last_cuda_error(e);
      return B2F_ERR_CUDA;
    }
    cache[dev] = p;
  }
  *out = cache[dev];
  return B2F_OK;
}

}  // namespace b2f

extern "C" int b2f_qkv_decode_attn_noalloc(const void* q, const uint8_t* k_pages, const float* k_scales,
                                           const uint8_t* v_pages, const float* v_scales,
                                           const int32_t* block_table, int64_t max_pages,
                                           const int32_t* seq_lens, int64_t B, int64_t Hq, int64_t Hkv,
                                           int64_t D, int64_t page_size, int64_t head_stride,
                                           int64_t slot_stride, int bits, int group_size,
                                           float softmax_scale, int n_splits, void* out, void* stream) {
  if (B <= 0 || Hq <= 0 || D <= 0 || n_splits < 1) {
    return b2f_qkv_decode_attn(q, k_pages, k_scales, v_pages, v_scales, block_table, max_pages, seq_lens, B,
                               Hq, Hkv, D, page_size, head_stride, slot_stride, bits, group_size,
                               softmax_scale, n_splits, nullptr, 0, out, stream);
  }
  const int64_t need = b2f_qkv_decode_attn_workspace_bytes(B, Hq, D, n_splits);
  if (need > int64_t(B2F_ATTN_NOALLOC_SCRATCH_BYTES)) return B2F_ERR_WORKSPACE;
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = b2f::attn_noalloc_scratch(&scratch);
    if (rc != B2F_OK) return rc;
  }
  return b2f_qkv_decode_attn(q, k_pages, k_scales, v_pages, v_scales, block_table, max_pages, seq_lens, B, Hq,
                             Hkv, D, page_size, head_stride, slot_stride, bits, group_size, softmax_scale,
                             n_splits, scratch, need, out, stream);
}
