// (c) grouped dequant GEMM for decode-sized expert tiles: warp-level tensor-core
// MMA (mma.sync m16n8k16, bf16 in, fp32 accumulate) on 4-bit codes unpacked in
// registers.  Same contract as b2f_gather_qgemm_affine_tcgen05
// (mx.gather_qmm, expert_streaming.py:230-241, with the SwitchGLU front half of
// kernels/ops.py:48-108 fused when w_up is given).
//
// Why this path exists next to the tcgen05 kernels: at decode a routed expert
// sees a handful of tokens (typically 1-16).  tcgen05.mma costs a fixed ~55
// cycles per M=128,K=16 instruction for every N <= 64 on B200 (measured), at
// most ~37 weights per cycle per SM against the ~44 weights per cycle per SM at
// which 4-bit weights stream from HBM, and its operands pass through shared
// memory as dequantized bf16.  mma.sync measures 554 TFLOP/s (bf16) on B200;
// with 16 weight rows as its M side and up to 8 tokens as its N side, each code
// is read once from shared memory and consumed from registers.
//
// Arithmetic (the order MLX's own quantized kernels use): per 64-wide group g
//   y[t, n] += s[n,g] * sum_k q[n,k] x[t,k] + b[n,g] * sum_k x[t,k]
// The codes enter the MMA as the exact bf16 values 128+q (one lop3 per pair),
// so the group sum is T = sum (128+q) x and y += s*T + (b - 128 s)*X with
// X = sum x, itself one MMA against an all-ones operand; everything after the
// bf16 products is fp32.
//
// CTA = 4 consumer warps + 1 producer warp.  Per 128-wide K chunk the producer
// TMA-loads the CTA's weight rows (64 bytes of codes per row, 64B-swizzled) and
// bulk-copies the slot's token rows (256 bytes each, stored 320 bytes apart so
// the consumers' 16-byte reads hit distinct banks) into a ring of S stages.
// Each consumer warp owns 64 weight rows (gate/up: 32 rows of each matrix).
//
// K mapping inside a chunk: lane (r = lane/4, c = lane%4), code word j (0..3)
// of a row covers k in [8c + 32j, 8c + 32j + 8); nibble i is k + i (MLX's
// LSB-first order).  MMA k-step 2j takes the nibble pairs (0,4) and (1,5) of
// word j, k-step 2j+1 the pairs (2,6) and (3,7), and the token fragments the
// same pairs; words 0-1 are group 2h of chunk h, words 2-3 group 2h+1.
#include "common.cuh"
#include "tc_common.cuh"

namespace b2f {

constexpr int MMA_CW = 4;         // consumer warps per CTA
// bytes between token rows of a staged x chunk (4-bit / 2-bit weights): 256
// bytes of a row plus padding that keeps the fragment reads conflict free
template <int BITS>
constexpr int mma_xstride() { return BITS == 4 ? 320 : 336; }

// Two shapes of the same kernel:
//   expert tiles (plan tile 16): slots of <= 16 tokens, 64 weight rows per
//     warp, three CTAs per SM;
//   expert tiles (plan tile 32): slots of <= 32 tokens, 32 weight rows per
//     warp, two CTAs per SM (168 registers): an expert routed 17-32 tokens
//     unpacks its codes once instead of twice (hot experts under skewed
//     routing);
//   wide tiles (plan tile 64, one matrix): slots of <= 64 tokens (a dense
//     projection of a decode batch is one slot), 16 weight rows per warp so
//     the rows spread over many CTAs, two CTAs per SM.
template <int TILE>
struct MmaShape;
template <>
struct MmaShape<16> {
  static constexpr int NTMAX = 2, WROWS = 64, CTAS = 3;
};
template <>
struct MmaShape<32> {
  static constexpr int NTMAX = 4, WROWS = 32, CTAS = 2;
};
template <>
struct MmaShape<64> {
  static constexpr int NTMAX = 8, WROWS = 16, CTAS = 2;
};


struct MmaParams {
  const __nv_bfloat16* x;
  int64_t ldx;
  const int32_t* x_row_index;
  int64_t x_row_div;
  const __nv_bfloat16* s[2];
  const __nv_bfloat16* b[2];
  int64_t N, K;
  int G;  // quantization groups per row (K / 64)
  __nv_bfloat16* out;
  int64_t ldo;
  int out_plan;  // 1: output rows in plan order, columns permuted (0,4,1,5,2,6,3,7) per 8
  const int32_t* slot_count;
  const int4* slots;
  const int32_t* sorted;
  int32_t* err;
  int stages;
  int cpk;         // 128-wide K chunks per split (grid z); the whole K when not split
  float* partial;  // split-K: fp32 planes [gridDim.z][A][N] instead of bf16 out (one matrix)
  int64_t plane;   // elements per partial plane (A * N)
  int slot_major;  // grid x = slot (the slots sharing a row block run back to back and hit L2)
  // packed weights (b2f_mma_repack): tile (expert, row block, chunk) at byte
  // ((expert * nb + row block) * (K/128) + chunk) * tile_bytes of pw[m]
  const uint8_t* pw[2];
  int64_t nb;
  // programmatic dependent launch: bit 0 = this launch depends on the kernel
  // before it in the stream, whose output is only the activation rows
  // (weights of the first ring stages are fetched, then griddepcontrol.wait,
  // then the activation rows; the plan is two or more launches old); bit 2 =
  // a programmatic launch that waits before anything else; bit 1 = let the
  // next kernel launch once every CTA of this one has waited (or, in a
  // normal launch, has started)
  int flags;
  // stream-K (packed tiles, one K range): fp32 partials, 2 x 4096 floats per
  // CTA, and one arrival counter per CTA (zero before the first launch; every
  // launch that completes leaves them zero); rb = row blocks per slot
  float* sk_part;
  int32_t* sk_cnt;
  int rb;
};


__device__ __forceinline__ void mma_bf16_16816_zero(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(0.f));
}

// (d0, d1) = (a0*b0 + c0, a1*b1 + c1), one packed fp32x2 FMA (two round-to-nearest FMAs)
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                      float c1) {
  unsigned long long a, b, c, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(b0), "f"(b1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(c) : "f"(c0), "f"(c1));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
// half `hi` of a pair of bf16 (or fp16) scale / bias values as fp32
template <bool F16>
__device__ __forceinline__ float sc_half(uint32_t v, int hi) {
  if constexpr (F16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(hi ? v >> 16 : v & 0xFFFFu)));
  } else {
    return hi ? bf_hi(v) : bf_lo(v);
  }
}

// Named barrier 1 over the MMA_CW consumer warps (the producer warp never
// takes it); consumers_or also returns whether any consumer passed non-zero.
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(MMA_CW * 32) : "memory"); }
__device__ __forceinline__ int consumers_or(int v) {
  int r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.s32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"(v), "n"(MMA_CW * 32)
      : "memory");
  return r;
}

// Stream-K cut of one item between two CTAs: each stores its fp32
// accumulators (thread-private layout, 4096 floats per partial) and counts
// itself in; the second to arrive adds the other's partial (fp32 addition
// commutes, so the sum does not depend on which arrives second), leaves the
// counter zero and runs the epilogue.
struct MmaCut {
  float* mine;
  const float* other;
  int32_t* counter;
};
// kind 1: the item's first chunks, this CTA's last item (its partial slot 1;
// the next CTA's slot 0, counter of this CTA); kind 2: the item's last
// chunks, this CTA's first item (slot 0; the previous CTA's slot 1 and counter)
__device__ __forceinline__ MmaCut mma_cut(const MmaParams& p, int kind) {
  const int64_t g = blockIdx.x;
  if (kind == 1) return {p.sk_part + (2 * g + 1) * 4096, p.sk_part + (2 * g + 2) * 4096, p.sk_cnt + g};
  return {p.sk_part + 2 * g * 4096, p.sk_part + (2 * g - 1) * 4096, p.sk_cnt + (g - 1)};
}

// The consumer side of one CTA for slots of up to 8*NTA tokens: the warp's
// WROWS/MAT rows of each matrix (MAT 2: gate and up, SwiGLU epilogue), as
// MT row tiles of 16.
template <int MAT, int NTA, bool XPLAN, int WROWS, int BITS, bool SF16, bool PACKED = false>
__device__ __forceinline__ int mma_consume(const MmaParams& p, uint8_t* smem, int STAGE, int W_BYTES, int CTA_ROWS,
                                            uint64_t* full, uint64_t* empty, volatile int* abort_flag, int expert,
                                            int begin, int cnt, int64_t row_base, int h0, int h1, int warp,
                                            int lane, int& s, uint32_t& phase, bool walk, int cut_kind,
                                            volatile int* sk_flag) {
  constexpr int MT = WROWS / 16 / MAT;
  static_assert(MT >= 1, "at least one 16-row tile per matrix");
  const int S = p.stages;
  const int r = lane >> 2, c = lane & 3;
  // swizzle phase of this lane's rows (r and r+8 share it): 64B (4-bit rows
  // of 64 bytes) or 32B (2-bit rows of 32 bytes)
  const int sw = BITS == 4 ? (r >> 1) & 3 : (r >> 2) & 1;
  constexpr int RBY = 16 * BITS;  // code bytes per row per 128-wide chunk
  constexpr int XS = mma_xstride<BITS>();
  const int wr0 = warp * (WROWS / MAT);
  const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};

  float acc[MAT][MT][NTA][4];
#pragma unroll
  for (int m = 0; m < MAT; ++m)
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int nt = 0; nt < NTA; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[m][i][nt][e] = 0.f;

  // (s, b) pairs of both groups of a chunk for rows R and R+8 of each tile
  uint32_t sr[MAT][MT][2], br[MAT][MT][2];
  // the pair of chunk h sits at 32-bit word h of a row (G is even); rows R
  // and R+8 of tile i are (2i + hf) * 4G words past the lane's first row
  const int64_t srow0 = (int64_t(expert) * p.N + row_base + wr0 + r) * p.G;
  const uint32_t* sbase[MAT];
  const uint32_t* bbase[MAT];
#pragma unroll
  for (int m = 0; m < MAT; ++m) {
    sbase[m] = reinterpret_cast<const uint32_t*>((m == 0 ? p.s[0] : p.s[1]) + srow0);
    bbase[m] = reinterpret_cast<const uint32_t*>((m == 0 ? p.b[0] : p.b[1]) + srow0);
  }
  const int rstep = 4 * p.G;
  const int64_t rows_left = p.N - (row_base + wr0 + r);  // rows valid at offsets < rows_left
  // matrix m's tile in a stage: codes (CTA_ROWS rows of RBY bytes), then for
  // packed tiles each row's 8 bytes of (s, s, b, b) for the chunk's 2 groups
  const int TB = CTA_ROWS * (RBY + (PACKED ? 8 : 0));
  auto load_sb = [&](int h) {
    if constexpr (PACKED) return;  // read from the stage once it has landed
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const bool rv = 16 * i + 8 * hf < rows_left;
        const int o = (2 * i + hf) * rstep + h;
#pragma unroll
        for (int m = 0; m < MAT; ++m) {
          sr[m][i][hf] = rv ? sbase[m][o] : 0u;
          br[m][i][hf] = rv ? bbase[m][o] : 0u;
        }
      }
  };
  load_sb(h0);

  // ring position (s, phase) carries over from the CTA's previous item
  for (int h = h0; h < h1; ++h) {
    const bool ok = !*abort_flag && mbar_wait_bounded(&full[s], phase);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) *abort_flag = 1;
      break;
    }
    const uint8_t* wst = smem + s * STAGE;
    const uint8_t* xst = wst + W_BYTES;
    if constexpr (PACKED) {
#pragma unroll
      for (int m = 0; m < MAT; ++m)
#pragma unroll
        for (int i = 0; i < MT; ++i)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const uint2 v = *reinterpret_cast<const uint2*>(wst + m * TB + CTA_ROWS * RBY +
                                                            (wr0 + 16 * i + 8 * hf + r) * 8);
            sr[m][i][hf] = v.x;
            br[m][i][hf] = v.y;
          }
    }
#pragma unroll
    for (int grp = 0; grp < 2; ++grp) {
      float t[MAT][MT][NTA][4];  // sum over the group of (128+q) x
      float xs[NTA][4];          // sum over the group of x (rows all equal)
      if constexpr (BITS == 2) {
        // 2-bit: word c + 4*grp of the row's 8-word chunk, 16 crumbs (LSB
        // first) covering k in [16(c + 4 grp), +16); crumb pairs (i, i+8)
        // through k-steps 0..3 as (0,8)(1,9) | (2,10)(3,11) | ...
        uint32_t bx[NTA][4][2];
#pragma unroll
        for (int nt = 0; nt < NTA; ++nt) {
          const uint8_t* xp = xst + (8 * nt + r) * XS + 32 * (c + 4 * grp);
          const uint4 u0 = *reinterpret_cast<const uint4*>(xp), u1 = *reinterpret_cast<const uint4*>(xp + 16);
          const uint32_t uu[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
          for (int st = 0; st < 4; ++st) {
            bx[nt][st][0] = prmt(uu[st], uu[st + 4], 0x5410u);  // (x 2st, x 2st+8)
            bx[nt][st][1] = prmt(uu[st], uu[st + 4], 0x7632u);  // (x 2st+1, x 2st+9)
            if (st == 0) {
              mma_bf16_16816_zero(xs[nt], ones, bx[nt][st]);
            } else {
              mma_bf16_16816(xs[nt], ones, bx[nt][st]);
            }
          }
        }
#pragma unroll
        for (int m = 0; m < MAT; ++m) {
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            const uint8_t* rowp = wst + m * TB + (wr0 + 16 * i + r) * RBY + 16 * (grp ^ sw) + 4 * c;
            const uint32_t wl = *reinterpret_cast<const uint32_t*>(rowp);
            const uint32_t wh = *reinterpret_cast<const uint32_t*>(rowp + 8 * RBY);
#pragma unroll
            for (int st = 0; st < 4; ++st) {
              const uint32_t a[4] = {and_or(wl >> (4 * st), 0x00030003u, 0x43004300u),
                                     and_or(wh >> (4 * st), 0x00030003u, 0x43004300u),
                                     and_or(wl >> (4 * st + 2), 0x00030003u, 0x43004300u),
                                     and_or(wh >> (4 * st + 2), 0x00030003u, 0x43004300u)};
#pragma unroll
              for (int nt = 0; nt < NTA; ++nt) {
                if (st == 0) {
                  mma_bf16_16816_zero(t[m][i][nt], a, bx[nt][st]);
                } else {
                  mma_bf16_16816(t[m][i][nt], a, bx[nt][st]);
                }
              }
            }
          }
        }
      } else {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int j = 2 * grp + jj;
        // token fragments: token 8nt + r, pairs (0,4) (1,5) | (2,6) (3,7)
        uint32_t bx[NTA][2][2];
#pragma unroll
        for (int nt = 0; nt < NTA; ++nt) {
          const uint4 u = *reinterpret_cast<const uint4*>(xst + (8 * nt + r) * XS + 16 * c + 64 * j);
          if constexpr (XPLAN) {  // stored as (0,4,1,5,2,6,3,7): the pairs already
            bx[nt][0][0] = u.x;
            bx[nt][0][1] = u.y;
            bx[nt][1][0] = u.z;
            bx[nt][1][1] = u.w;
          } else {
            bx[nt][0][0] = prmt(u.x, u.z, 0x5410u);
            bx[nt][0][1] = prmt(u.x, u.z, 0x7632u);
            bx[nt][1][0] = prmt(u.y, u.w, 0x5410u);
            bx[nt][1][1] = prmt(u.y, u.w, 0x7632u);
          }
          if (jj == 0) {
            mma_bf16_16816_zero(xs[nt], ones, bx[nt][0]);
          } else {
            mma_bf16_16816(xs[nt], ones, bx[nt][0]);
          }
          mma_bf16_16816(xs[nt], ones, bx[nt][1]);
        }
#pragma unroll
        for (int m = 0; m < MAT; ++m) {
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            const uint8_t* rowp = wst + m * TB + (wr0 + 16 * i + r) * 64 + 16 * (j ^ sw) + 4 * c;
            const uint32_t wl = *reinterpret_cast<const uint32_t*>(rowp);
            const uint32_t wh = *reinterpret_cast<const uint32_t*>(rowp + 8 * 64);
            const uint32_t a0[4] = {and_or(wl, 0x000F000Fu, 0x43004300u), and_or(wh, 0x000F000Fu, 0x43004300u),
                                    and_or(wl >> 4, 0x000F000Fu, 0x43004300u),
                                    and_or(wh >> 4, 0x000F000Fu, 0x43004300u)};
            const uint32_t a1[4] = {and_or(wl >> 8, 0x000F000Fu, 0x43004300u),
                                    and_or(wh >> 8, 0x000F000Fu, 0x43004300u),
                                    and_or(wl >> 12, 0x000F000Fu, 0x43004300u),
                                    and_or(wh >> 12, 0x000F000Fu, 0x43004300u)};
#pragma unroll
            for (int nt = 0; nt < NTA; ++nt) {
              if (jj == 0) {
                mma_bf16_16816_zero(t[m][i][nt], a0, bx[nt][0]);
              } else {
                mma_bf16_16816(t[m][i][nt], a0, bx[nt][0]);
              }
              mma_bf16_16816(t[m][i][nt], a1, bx[nt][1]);
            }
          }
        }
      }
      }
      // fold the group: y += s*T + (b - 128 s)*X   (rows R: e 0,1; R+8: e 2,3)
#pragma unroll
      for (int m = 0; m < MAT; ++m)
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          const float s0 = sc_half<SF16>(sr[m][i][0], grp), s1 = sc_half<SF16>(sr[m][i][1], grp);
          const float c0 = fmaf(-128.f, s0, sc_half<SF16>(br[m][i][0], grp));
          const float c1 = fmaf(-128.f, s1, sc_half<SF16>(br[m][i][1], grp));
#pragma unroll
          for (int nt = 0; nt < NTA; ++nt) {
            // (rows R, R+8) x (tokens 2c, 2c+1) as two packed pairs: the same
            // round-to-nearest FMAs as one scalar FMA per element
            float* a = acc[m][i][nt];
            ffma2(a[0], a[1], c0, c0, xs[nt][0], xs[nt][1], a[0], a[1]);
            ffma2(a[0], a[1], s0, s0, t[m][i][nt][0], t[m][i][nt][1], a[0], a[1]);
            ffma2(a[2], a[3], c1, c1, xs[nt][0], xs[nt][1], a[2], a[3]);
            ffma2(a[2], a[3], s1, s1, t[m][i][nt][2], t[m][i][nt][3], a[2], a[3]);
          }
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (h + 1 < h1) load_sb(h + 1);
    if (++s == S) {
      s = 0;
      phase ^= 1u;
    }
  }
  if (!walk) {
    if (*abort_flag) return 1;
  } else {
    // a CTA walking several items: every consumer warp takes the same path
    // (the next item's barriers need all of them)
    if (consumers_or(*abort_flag)) return 1;
    if (cut_kind) {
      const MmaCut cut = mma_cut(p, cut_kind);
      const int tid = threadIdx.x;  // consumer threads are 0 .. 32*MMA_CW-1
      int k = 0;
#pragma unroll
      for (int m = 0; m < MAT; ++m)
#pragma unroll
        for (int i = 0; i < MT; ++i)
#pragma unroll
          for (int nt = 0; nt < NTA; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) __stcg(cut.mine + (k++) * (32 * MMA_CW) + tid, acc[m][i][nt][e]);
      consumers_sync();
      if (tid == 0) {
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        const int old = atomicAdd(cut.counter, 1);
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        if (old) *cut.counter = 0;
        *sk_flag = old;
      }
      consumers_sync();
      if (*sk_flag == 0) return 0;  // the other CTA finishes the item
      k = 0;
#pragma unroll
      for (int m = 0; m < MAT; ++m)
#pragma unroll
        for (int i = 0; i < MT; ++i)
#pragma unroll
          for (int nt = 0; nt < NTA; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[m][i][nt][e] += __ldcg(cut.other + (k++) * (32 * MMA_CW) + tid);
    }
  }

  if (p.partial) {
    // split-K: fp32 partial plane of this K range, rows = assignments
    float* plane = p.partial + int64_t(blockIdx.z) * p.plane;
#pragma unroll
    for (int nt = 0; nt < NTA; ++nt) {
      const int t0 = 8 * nt + 2 * c;
      const int64_t a0 = t0 < cnt ? int64_t(p.sorted[begin + t0]) : 0;
      const int64_t a1 = t0 + 1 < cnt ? int64_t(p.sorted[begin + t0 + 1]) : 0;
#pragma unroll
      for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const float v0 = acc[0][i][nt][2 * hf], v1 = acc[0][i][nt][2 * hf + 1];
          const int64_t row8 = row_base + wr0 + 16 * i + 8 * hf;
          const float recv = __shfl_xor_sync(0xffffffffu, (r & 1) ? v0 : v1, 4);
          const bool odd = r & 1;
          const int tok = odd ? t0 + 1 : t0;
          const int64_t col = row8 + (r & ~1);
          if (tok < cnt && col < p.N)
            *reinterpret_cast<float2*>(plane + (odd ? a1 : a0) * p.N + col) =
                odd ? make_float2(recv, v1) : make_float2(v0, recv);
        }
    }
    return 0;
  }

  // ---- epilogue: values (row R or R+8, tokens 2c and 2c+1) -> bf16 rows ------
#pragma unroll
  for (int nt = 0; nt < NTA; ++nt) {
    const int t0 = 8 * nt + 2 * c;
    int64_t orow0 = 0, orow1 = 0;
    if (t0 < cnt) orow0 = p.out_plan ? int64_t(begin + t0) : int64_t(p.sorted[begin + t0]);
    if (t0 + 1 < cnt) orow1 = p.out_plan ? int64_t(begin + t0 + 1) : int64_t(p.sorted[begin + t0 + 1]);
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float v0 = acc[0][i][nt][2 * hf], v1 = acc[0][i][nt][2 * hf + 1];
        if constexpr (MAT == 2) {
          v0 = silu_mul_tc(v0, acc[1][i][nt][2 * hf]);
          v1 = silu_mul_tc(v1, acc[1][i][nt][2 * hf + 1]);
        }
        const int64_t row8 = row_base + wr0 + 16 * i + 8 * hf;  // first row of this lane's 8-row group
        if (!p.out_plan) {
          // lanes r and r^1 trade so each holds two adjacent rows of one token
          const float recv = __shfl_xor_sync(0xffffffffu, (r & 1) ? v0 : v1, 4);
          const bool odd = r & 1;
          const int tok = odd ? t0 + 1 : t0;
          const int64_t col = row8 + (r & ~1);
          if (tok < cnt && col < p.N)
            *reinterpret_cast<uint32_t*>(p.out + (odd ? orow1 : orow0) * p.ldo + col) =
                odd ? pack_bf16x2(recv, v1) : pack_bf16x2(v0, recv);
        } else {
          // (0,4,1,5,2,6,3,7) order: lanes r and r^4 trade, positions 2(r&3), 2(r&3)+1
          const bool up = r >= 4;
          const float recv = __shfl_xor_sync(0xffffffffu, up ? v0 : v1, 16);
          const int tok = up ? t0 + 1 : t0;
          if (tok < cnt && row8 < p.N)
            *reinterpret_cast<uint32_t*>(p.out + (up ? orow1 : orow0) * p.ldo + row8 + 2 * (r & 3)) =
                up ? pack_bf16x2(recv, v1) : pack_bf16x2(v0, recv);
        }
      }
  }
  return 0;
}

template <int MAT, bool XPLAN, int TILE, int BITS = 4, bool SF16 = false, bool PACKED = false, bool WALK = false>
__global__ void __launch_bounds__(160, MmaShape<TILE>::CTAS)
    qgemm_mma_kernel(const MmaParams p, const __grid_constant__ CUtensorMap tm0,
                     const __grid_constant__ CUtensorMap tm1) {
  using SH = MmaShape<TILE>;
  constexpr int CTA_ROWS = MMA_CW * SH::WROWS / MAT;  // weight rows per matrix
  constexpr int RBY = 16 * BITS;                      // code bytes per row per chunk
  constexpr int XS = mma_xstride<BITS>();             // token row pitch in a stage
  constexpr int TB = CTA_ROWS * (RBY + (PACKED ? 8 : 0));  // one matrix's tile (packed: + scales)
  constexpr int W_BYTES = MAT * TB;
  constexpr int STAGE = (W_BYTES + TILE * XS + 1023) / 1024 * 1024;

  extern __shared__ __align__(1024) uint8_t mma_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(mma_smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * STAGE);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);

  volatile int* sk_flag = abort_flag + 1;
  int64_t* sk_range = reinterpret_cast<int64_t*>(const_cast<int*>(abort_flag + 2));  // stream-K [u0, u1)

  if (p.flags & 4) pdl_wait();
  if ((p.flags & 2) && !(p.flags & 1) && threadIdx.x == 0) pdl_trigger();
  // bit 0: a CTA without work still waits, so the grid never completes
  // before the kernel it depends on
  const bool idle_wait = (p.flags & 1) != 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HC = int(p.K >> 7);

  // The CTA's items: (slot, row block) pairs, each with a K chunk range.
  // Per-item grid: x = row block, y = slot (one expert's contiguous rows are
  // streamed by consecutive CTAs; slot-major -- wide tiles, one-matrix plans
  // -- x = slot, so the slots reading one row block run back to back and
  // share it in L2), z = K range.  Stream-K (p.sk_part): the live items in
  // (slot, row block) order times their HC chunks are cut into G equal unit
  // ranges, G = min(grid, live items), so a range spans >= HC units and an
  // item is cut between at most two CTAs.
  constexpr bool walk = WALK;  // stream-K: p.sk_part is set
  int n_it = 1;
  int one_slot = 0, one_rblk = 0, one_h0 = 0, one_h1 = 0;
  if (walk) {
    const int64_t n_items = int64_t(*p.slot_count) * p.rb;
    const int64_t G = min(int64_t(gridDim.x), n_items);
    if (int64_t(blockIdx.x) >= G) {
      if (idle_wait) pdl_wait();
      return;
    }
    const int64_t U = n_items * HC;
    const int64_t u0 = int64_t(blockIdx.x) * U / G, u1 = (int64_t(blockIdx.x) + 1) * U / G;
    n_it = int((u1 - 1) / HC - u0 / HC + 1);
    if (threadIdx.x == 0) {
      sk_range[0] = u0;
      sk_range[1] = u1;
    }
  } else {
    one_slot = p.slot_major ? int(blockIdx.x) : int(blockIdx.y);
    one_rblk = p.slot_major ? int(blockIdx.y) : int(blockIdx.x);
    one_h0 = int(blockIdx.z) * p.cpk;
    one_h1 = min(HC, one_h0 + p.cpk);
    bool idle = one_slot >= *p.slot_count || int64_t(one_rblk) * CTA_ROWS >= p.N || one_h0 >= one_h1;
    if (!idle) idle = p.slots[one_slot].z <= 0;
    if (idle) {
      if (idle_wait) pdl_wait();
      return;
    }
  }
  struct Item {
    int expert, begin, cnt, rblk, h0, h1;
    int64_t row_base;
    int cut;  // 0 whole; 1 its first chunks (this CTA's last item); 2 its last chunks (this CTA's first item)
  };
  auto item_at = [&](int ii) {
    Item w;
    int slot;
    if (walk) {
      const int64_t u0 = sk_range[0], u1 = sk_range[1];
      const int64_t i = u0 / HC + ii;
      slot = int(i / p.rb);
      w.rblk = int(i - int64_t(slot) * p.rb);
      w.h0 = int(max(u0 - i * HC, int64_t(0)));
      w.h1 = int(min(u1 - i * HC, int64_t(HC)));
      w.cut = w.h0 > 0 ? 2 : (w.h1 < HC ? 1 : 0);
    } else {
      slot = one_slot;
      w.rblk = one_rblk;
      w.h0 = one_h0;
      w.h1 = one_h1;
      w.cut = 0;
    }
    const int4 sl = p.slots[slot];
    w.expert = sl.x;
    w.begin = sl.y;
    w.cnt = min(sl.z, TILE);
    w.row_base = int64_t(w.rblk) * CTA_ROWS;
    return w;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], MMA_CW);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == MMA_CW) {
    // ---- producer: weight tiles by TMA, one token row per lane by bulk copy ----
    if (producers_stalled()) {  // test control: nothing is issued, the consumers' waits run out
      if (idle_wait) pdl_wait();
      return;
    }
    constexpr int XPL = (TILE + 31) / 32;  // token rows per producer lane
    const __nv_bfloat16* xrow[XPL];
    auto issue_weights = [&](const Item& w, int hh, uint8_t* st, uint64_t* bar) {
      if constexpr (PACKED) {
        // the tile is stored as its shared-memory image: one contiguous copy per matrix
        const int64_t off = ((int64_t(w.expert) * p.nb + w.rblk) * (p.K >> 7) + hh) * int64_t(TB);
        bulk_g2s(st, p.pw[0] + off, uint32_t(TB), bar);
        if constexpr (MAT == 2) bulk_g2s(st + TB, p.pw[1] + off, uint32_t(TB), bar);
      } else {
        const int wrow = int(int64_t(w.expert) * p.N + w.row_base);
        tma_load_2d(st, &tm0, hh * (4 * BITS), wrow, bar);
        if constexpr (MAT == 2) tma_load_2d(st + CTA_ROWS * RBY, &tm1, hh * (4 * BITS), wrow, bar);
      }
    };
    auto issue_x = [&](const Item& w, int hh, uint8_t* st, uint64_t* bar) {
#pragma unroll
      for (int u = 0; u < XPL; ++u) {
        const int tk = lane + 32 * u;
        if (tk < w.cnt) bulk_g2s(st + W_BYTES + tk * XS, xrow[u] + int64_t(hh) * 128, 256u, bar);
      }
    };
    int s = 0;
    uint32_t phase = 0;
    int64_t issued = 0;
    bool stop = false;
    for (int ii = 0; ii < n_it && !stop; ++ii) {
      const Item w = item_at(ii);
#pragma unroll
      for (int u = 0; u < XPL; ++u) {
        xrow[u] = nullptr;
        const int tk = lane + 32 * u;
        if (tk < w.cnt) {
          const int pos = w.begin + tk;
          int64_t row;
          if constexpr (XPLAN) {
            row = pos;
          } else {
            const int a = p.sorted[pos];
            row = p.x_row_index ? int64_t(p.x_row_index[a]) : int64_t(a) / p.x_row_div;
          }
          xrow[u] = p.x + row * p.ldx;
        }
      }
      const uint32_t tx = uint32_t(W_BYTES + w.cnt * 256);
      int h = w.h0;
      if (ii == 0 && (p.flags & 1)) {
        // dependent launch: the first stages' weights need nothing from the kernel
        // before this one, so they are in flight before the wait; the activation
        // rows (that kernel's output) are copied after it
        const int pre = min(S, w.h1 - w.h0);
        if (lane == 0)
          for (int u = 0; u < pre; ++u) {
            mbar_arrive_expect_tx(&full[u], tx);
            issue_weights(w, w.h0 + u, smem + u * STAGE, &full[u]);
          }
        __syncwarp();
        pdl_wait();
        if ((p.flags & 2) && lane == 0) pdl_trigger();
        for (int u = 0; u < pre; ++u) issue_x(w, w.h0 + u, smem + u * STAGE, &full[u]);
        h += pre;
        issued = pre;
        s = pre % S;
        phase = pre == S ? 1u : 0u;
      }
      for (; h < w.h1; ++h) {
        int ok = 1;
        if (lane == 0) {
          if (issued >= S && !mbar_wait_bounded_backoff(&empty[s], phase ^ 1u)) ok = 0;
          if (*abort_flag) ok = 0;
          if (ok) {
            mbar_arrive_expect_tx(&full[s], tx);
          } else {
            *abort_flag = 1;
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          stop = true;
          break;
        }
        uint8_t* st = smem + s * STAGE;
        if (lane == 0) issue_weights(w, h, st, &full[s]);
        issue_x(w, h, st, &full[s]);
        ++issued;
        if (++s == S) {
          s = 0;
          phase ^= 1u;
        }
      }
    }
    // copies already issued land before the CTA goes away
    if (lane == 0)
      for (int64_t k = 1; k <= S && issued - k >= 0; ++k)
        mbar_wait_bounded(&full[(issued - k) % S], uint32_t(((issued - k) / S) & 1), 100000000ull);
    return;
  }

  int s = 0;
  uint32_t phase = 0;
  for (int ii = 0; ii < n_it; ++ii) {
    const Item w = item_at(ii);
    int ab;
#define B2F_MMA_CONSUME(NT)                                                                                         \
  mma_consume<MAT, NT, XPLAN, SH::WROWS, BITS, SF16, PACKED>(p, smem, STAGE, W_BYTES, CTA_ROWS, full, empty,       \
                                                             abort_flag, w.expert, w.begin, w.cnt, w.row_base,    \
                                                             w.h0, w.h1, warp, lane, s, phase, walk, w.cut, sk_flag)
    if constexpr (SH::NTMAX == 2) {
      ab = w.cnt <= 8 ? B2F_MMA_CONSUME(1) : B2F_MMA_CONSUME(2);
    } else if constexpr (SH::NTMAX == 4) {
      ab = w.cnt <= 8 ? B2F_MMA_CONSUME(1) : (w.cnt <= 16 ? B2F_MMA_CONSUME(2) : B2F_MMA_CONSUME(4));
    } else {
      ab = B2F_MMA_CONSUME(SH::NTMAX);
    }
#undef B2F_MMA_CONSUME
    if (ab) break;
  }
  if (lane == 0 && *abort_flag) report_timeout(p.err);
}

// Code rows as a 2-D uint32 tensor [rows, K*bits/32]; box = one 128-wide K
// chunk (4-bit: 16 words = 64 bytes, 64B swizzle; 2-bit: 8 words = 32
// bytes, 32B swizzle) of `box_rows` rows.
static int make_mma_weight_map(CUtensorMap* map, const uint32_t* w, int64_t rows, int64_t K, int box_rows,
                               int bits = 4) {
  const cuuint64_t words = cuuint64_t(K * bits / 32);
  const cuuint64_t dims[2] = {words, cuuint64_t(rows)};
  const cuuint64_t strides[1] = {words * 4};
  const cuuint32_t box[2] = {cuuint32_t(4 * bits), cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(w), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, bits == 4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B2F_OK : B2F_ERR_INVALID;
}

template <int MAT, bool XPLAN, int TILE, int BITS = 4, bool SF16 = false, bool PACKED = false>
static int launch_mma_cfg(MmaParams p, const uint32_t* w0, const uint32_t* w1, int64_t E, int64_t slots_grid,
                          int ksplit, cudaStream_t st) {
  using SH = MmaShape<TILE>;
  constexpr int CTA_ROWS = MMA_CW * SH::WROWS / MAT;
  constexpr int STAGE = (MAT * CTA_ROWS * (16 * BITS + (PACKED ? 8 : 0)) + TILE * mma_xstride<BITS>() + 1023) / 1024 * 1024;
  // as many ring stages as fit in the CTA's share of the SM's 228 KB (1 KB
  // of it reserved per CTA); a grid that fits one CTA per SM (a decode step
  // of a few tokens) gives each CTA the whole SM's shared memory, so more
  // bytes are in flight per CTA
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                    cudaSuccess)
      sms = 148;
  }
  const int64_t row_blocks_all = (p.N + CTA_ROWS - 1) / CTA_ROWS;
  const int per_sm = slots_grid * row_blocks_all * ksplit <= sms ? 1 : SH::CTAS;
  int S = 8;
  while (S > 2 && per_sm * (S * STAGE + 1024 + 256 + 1024) > 228 * 1024) --S;
  p.stages = S;
  const int smem = S * STAGE + 1024 + 256;
  CUtensorMap m0{}, m1{};
  if constexpr (!PACKED) {
    int rc = make_mma_weight_map(&m0, w0, E * p.N, p.K, CTA_ROWS, BITS);
    if (rc != B2F_OK) return rc;
    if (w1) {
      rc = make_mma_weight_map(&m1, w1, E * p.N, p.K, CTA_ROWS, BITS);
      if (rc != B2F_OK) return rc;
    } else {
      m1 = m0;
    }
  }
  auto kern = qgemm_mma_kernel<MAT, XPLAN, TILE, BITS, SF16, PACKED, false>;
  if constexpr (PACKED) {
    if (p.sk_part) kern = qgemm_mma_kernel<MAT, XPLAN, TILE, BITS, SF16, PACKED, true>;
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return B2F_ERR_CUDA;
  }
  const int64_t row_blocks = (p.N + CTA_ROWS - 1) / CTA_ROWS;
  // wide tiles, and one-matrix plans whose slots all read the same rows, put
  // the slots on x; expert tiles keep one expert's row blocks consecutive
  p.slot_major = (TILE == 64 || E == 1) ? 1 : 0;
  if ((p.slot_major ? row_blocks : slots_grid) > 65535) return B2F_ERR_UNSUPPORTED;
  dim3 grid = p.slot_major ? dim3{unsigned(slots_grid), unsigned(row_blocks), unsigned(ksplit)}
                           : dim3{unsigned(row_blocks), unsigned(slots_grid), unsigned(ksplit)};
  if (p.sk_part) {
    // stream-K: one CTA per resident slot (at most the items of the plan's
    // largest slot count); the workspace holds sms * CTAS CTAs' partials
    if (ksplit != 1 || p.partial) return B2F_ERR_INVALID;
    p.rb = int(row_blocks);
    const int64_t items = slots_grid * row_blocks;
    grid = dim3{unsigned(min(int64_t(sms) * per_sm, items)), 1u, 1u};
  }
  // programmatic dependent launch (bit 0, or the thread's launch policy):
  // the grid may start while the previous kernel in the stream finishes.
  // Bit 0 prefetches weights before griddepcontrol.wait; otherwise every
  // thread waits first (bit 2).  Under the policy the next kernel may be
  // scheduled once every CTA has waited (bit 1).
  if (launch_pdl_policy()) p.flags |= 2;
  if (launch_pdl_policy() && !(p.flags & 1)) p.flags |= 4;
  if (p.flags & 5) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3{160, 1, 1};
    cfg.dynamicSmemBytes = size_t(smem);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, kern, p, m0, m1);
    if (le != cudaSuccess) {
      set_last_cuda_error(le);
      return B2F_ERR_CUDA;
    }
    return check_launch();
  }
  kern<<<grid, 160, smem, st>>>(p, m0, m1);
  return check_launch();
}

// Packed expert weights for the warp-MMA GEMM: 4-bit codes [E*N rows, K/8
// words] (MLX layout) with their bf16 scales / biases [E*N, K/64] -> per
// (expert, row block of `cr` rows, 128-wide K chunk) one tile of 72*cr bytes
// holding exactly the stage image the consumers read: first the codes as a
// 64B-swizzled TMA box of the tile would give them (row r at byte 64r, its
// 16-byte word group j at position j ^ ((r >> 1) & 3)), then per row 8 bytes
// (s[2h], s[2h+1], b[2h], b[2h+1]) for the chunk's two groups.  Rows past N
// are zero.  The producer fetches a whole tile with one contiguous bulk copy
// and the consumers take scales and biases from shared memory.
__global__ void __launch_bounds__(256) mma_repack_kernel(const uint32_t* __restrict__ wq,
                                                         const uint16_t* __restrict__ sc,
                                                         const uint16_t* __restrict__ bi, int64_t E, int64_t N,
                                                         int64_t K, int cr, int64_t nb, uint4* __restrict__ out) {
  const int hc = int(K >> 7);
  const int G = int(K >> 6);
  const int per_tile = cr * 4 + cr / 2;  // 16-byte groups: codes, then scales/biases (2 rows per group)
  const int64_t groups = E * nb * hc * per_tile;
  for (int64_t o = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; o < groups;
       o += int64_t(gridDim.x) * blockDim.x) {
    const int q = int(o % per_tile);
    int64_t t = o / per_tile;
    const int h = int(t % hc);
    t /= hc;
    const int64_t rb = t % nb;
    const int64_t e = t / nb;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (q < cr * 4) {
      const int rr = q >> 2, pos = q & 3;
      const int64_t row = rb * cr + rr;
      const int jj = pos ^ ((rr >> 1) & 3);
      if (row < N) v = reinterpret_cast<const uint4*>(wq + (e * N + row) * (K / 8) + int64_t(h) * 16)[jj];
    } else {
      uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int64_t row = rb * cr + 2 * (q - cr * 4) + u;
        if (row < N) {
          const int64_t g0 = (e * N + row) * G + 2 * h;
          w[2 * u] = uint32_t(sc[g0]) | (uint32_t(sc[g0 + 1]) << 16);
          w[2 * u + 1] = uint32_t(bi[g0]) | (uint32_t(bi[g0 + 1]) << 16);
        }
      }
      v = make_uint4(w[0], w[1], w[2], w[3]);
    }
    out[o] = v;
  }
}

// K split into ranges of whole 128-wide chunks: the number of non-empty ranges
static int mma_splitk_ranges(int64_t K, int ksplit, int* cpk) {
  const int hc = int(K / 128);
  if (ksplit < 1) ksplit = 1;
  if (ksplit > hc) ksplit = hc;
  *cpk = (hc + ksplit - 1) / ksplit;
  return (hc + *cpk - 1) / *cpk;
}

// plan layout helpers live in qgemv.cu
int64_t plan_slots_offset(int64_t A, int64_t E, int tile);
int64_t plan_sorted_offset(int64_t A, int64_t E, int tile);


// ---------------------------------------------------------------------------
// Dense projection of a decode batch: mx.quantized_matmul of M <= 64 token
// rows (the QuantizedLinear forward, layer_quantization.py:240-256 -- the
// q/k/v and o projections of a decode step) on warp MMA with the weights
// dequantized in registers.
//
// Work: units (128-row block, 128-wide K chunk) in row-block-major order,
// cut into G equal contiguous ranges (stream-K), G = the SM count or the unit
// count if smaller, so every SM streams the same number of weight tiles
// whatever N and K are.  A range ends in at most a few row blocks; each
// (row block, range) piece is summed in registers and stored as fp32 into
// plane `piece` of the output planes [P][M][N] -- piece = the range's index
// among the ranges covering that row block -- and the range that finishes a
// row block writes zeros into its remaining planes, so the P planes summed
// in plane order give the product with no atomics.
//
// CTA = 8 consumer warps (16 weight rows each) + 1 producer warp, one CTA
// per SM.  Per unit the producer TMA-loads the 128 rows' codes (64 bytes per
// row, 64B swizzle)
// and the token rows' 128 columns of x as one box of 160 columns x 64 rows
// (rows past M and columns past K arrive as zeros) into a ring stage -- two
// copies per unit, not one per token row; the 32 extra columns give the
// staged rows a 320-byte pitch, so the 16-byte fragment reads of 8 rows hit
// distinct banks.  Consumer lane (r, c) reads code word 4j + c of rows r and r+8 (k in [32j + 8c, +8)),
// turns each nibble pair (i, i+4) into the exact bf16 q as (128 + q) - 128,
// dequantizes w = q*s + b with one bf16 rounding (as the tcgen05 kernels do:
// no per-group fold, so the accumulators of all 64 tokens fit in registers)
// and multiplies with the token fragments of the same pairs.
constexpr int DEC_CW = 8;      // consumer warps per CTA (16 weight rows each)
constexpr int DEC_ROWS = 16 * DEC_CW;  // weight rows per CTA
constexpr int DEC_W = DEC_ROWS * 64;
constexpr int DEC_XS = 320;       // bytes between staged token rows (a 160-column box row)
constexpr int DEC_STAGE = DEC_W + 64 * DEC_XS;  // 24 KB
constexpr int DEC_CTAS = 1;     // CTAs per SM
constexpr int DEC_STAGES = 6;

struct DecParams {
  const __nv_bfloat16* x;
  int64_t ldx;
  int M;
  const uint32_t* sc;  // bf16 scales [N][G] as 32-bit words (groups 2h, 2h+1)
  const uint32_t* bi;
  int64_t N;
  int G;    // groups per row
  int C;    // 128-wide chunks per row
  int64_t U;  // units = row blocks * C
  int P;    // planes
  float* partial;  // [P][M][N]
  int stages;
};

// the CTA whose range holds unit u (ranges [g*U/G, (g+1)*U/G))
__host__ __device__ __forceinline__ int64_t dec_range_of(int64_t u, int64_t U, int64_t G) {
  return ((u + 1) * G - 1) / U;
}

template <int NT>
__device__ __forceinline__ void dec_store(const DecParams& p, float (&acc)[8][4], int plane, int64_t row_base,
                                          int warp, int r, int c, bool zero) {
  float* out = p.partial + int64_t(plane) * p.M * p.N;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int t0 = 8 * nt + 2 * c;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const float v0 = zero ? 0.f : acc[nt][2 * hf], v1 = zero ? 0.f : acc[nt][2 * hf + 1];
      // lanes r and r^1 trade so each holds two adjacent rows of one token
      const float recv = __shfl_xor_sync(0xffffffffu, (r & 1) ? v0 : v1, 4);
      const bool odd = r & 1;
      const int tok = odd ? t0 + 1 : t0;
      const int64_t col = row_base + 16 * warp + 8 * hf + (r & ~1);
      if (tok < p.M && col < p.N)
        *reinterpret_cast<float2*>(out + int64_t(tok) * p.N + col) =
            odd ? make_float2(recv, v1) : make_float2(v0, recv);
    }
  }
}

template <int NT>
__global__ void __launch_bounds__(32 * (DEC_CW + 1), DEC_CTAS) qgemm_decode_kernel(const DecParams p,
                                                                     const __grid_constant__ CUtensorMap tm,
                                                                     const __grid_constant__ CUtensorMap tmx) {
  extern __shared__ __align__(1024) uint8_t dec_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dec_smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * DEC_STAGE);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t G = gridDim.x, g = blockIdx.x;
  const int64_t u0 = g * p.U / G, u1 = (g + 1) * p.U / G;
  const int n_units = int(u1 - u0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], DEC_CW);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  const uint32_t tx = uint32_t(DEC_STAGE);  // the x boxes always carry 64 rows (zeros past M)

  if (warp == DEC_CW) {
    // ---- producer: the first stages' weights before waiting for the kernel
    // that writes x, then x rows and the rest of the ring ----
    const bool stalled = producers_stalled();  // test control: nothing is issued
    const int pre = min(S, n_units);
    if (lane == 0 && !stalled)
      for (int i = 0; i < pre; ++i) {
        const int64_t u = u0 + i;
        mbar_arrive_expect_tx(&full[i], tx);
        tma_load_2d(smem + i * DEC_STAGE, &tm, int(u % p.C) * 16, int((u / p.C) * DEC_ROWS), &full[i]);
      }
    pdl_wait();
    pdl_trigger();
    if (stalled) return;
    int issued = 0;
    for (int i = 0; i < n_units; ++i) {
      const int st = i % S;
      const int64_t u = u0 + i;
      const int h = int(u % p.C);
      if (i >= pre) {
        int ok = 1;
        if (lane == 0) {
          if (!mbar_wait_bounded_backoff(&empty[st], uint32_t(((i / S) - 1) & 1)) || *abort_flag) {
            *abort_flag = 1;
            ok = 0;
          } else {
            mbar_arrive_expect_tx(&full[st], tx);
            tma_load_2d(smem + st * DEC_STAGE, &tm, h * 16, int((u / p.C) * DEC_ROWS), &full[st]);
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      }
      if (lane == 0) tma_load_2d(smem + st * DEC_STAGE + DEC_W, &tmx, h * 128, 0, &full[st]);
      __syncwarp();
      issued = i + 1;
    }
    // copies already issued land before the CTA goes away
    if (lane == 0)
      for (int k = 1; k <= S && issued - k >= 0; ++k)
        mbar_wait_bounded(&full[(issued - k) % S], uint32_t(((issued - k) / S) & 1), 100000000ull);
    return;
  }

  pdl_wait();
  pdl_trigger();
  const int r = lane >> 2, c = lane & 3;
  const int sw = (r >> 1) & 3;  // 64B swizzle phase of rows r and r+8
  float acc[8][4];
  int64_t u = u0;
  int i = 0;
  bool aborted = false;
  while (u < u1 && !aborted) {
    const int64_t blk = u / p.C;
    const int64_t seg_end = min(u1, (blk + 1) * p.C);
    const int64_t row_base = blk * DEC_ROWS;
    const int64_t R0 = row_base + 16 * warp + r, R1 = R0 + 8;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
    // this segment's (s, b) of rows R0 and R1 for chunk h (groups 2h, 2h+1),
    // loaded one unit ahead of their use
    auto load_sb = [&](int64_t uu, uint32_t (&v)[4]) {
      const int hh = int(uu % p.C);
      v[0] = R0 < p.N ? p.sc[R0 * (p.G / 2) + hh] : 0u;
      v[1] = R0 < p.N ? p.bi[R0 * (p.G / 2) + hh] : 0u;
      v[2] = R1 < p.N ? p.sc[R1 * (p.G / 2) + hh] : 0u;
      v[3] = R1 < p.N ? p.bi[R1 * (p.G / 2) + hh] : 0u;
    };
    uint32_t sbn[4];
    load_sb(u, sbn);
    for (; u < seg_end; ++u, ++i) {
      const uint32_t s0 = sbn[0], b0 = sbn[1], s1 = sbn[2], b1 = sbn[3];
      if (u + 1 < seg_end) load_sb(u + 1, sbn);
      const int st = i % S;
      const bool ok = !*abort_flag && mbar_wait_bounded(&full[st], uint32_t((i / S) & 1));
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) *abort_flag = 1;
        aborted = true;
        break;
      }
      const uint8_t* wst = smem + st * DEC_STAGE;
      const uint8_t* xst = wst + DEC_W;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t sel = (j >> 1) ? 0x3232u : 0x1010u;  // group 2h + j/2 as a (v, v) pair
        const uint32_t S0 = prmt(s0, s0, sel), B0 = prmt(b0, b0, sel);
        const uint32_t S1 = prmt(s1, s1, sel), B1 = prmt(b1, b1, sel);
        const uint8_t* rowp = wst + (16 * warp + r) * 64 + 16 * (j ^ sw) + 4 * c;
        const uint32_t wl = *reinterpret_cast<const uint32_t*>(rowp);
        const uint32_t wh = *reinterpret_cast<const uint32_t*>(rowp + 8 * 64);
        uint32_t al[4], ah[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          al[q] = hfma2_bf(hsub2_bf(and_or(wl >> (4 * q), 0x000F000Fu, 0x43004300u), 0x43004300u), S0, B0);
          ah[q] = hfma2_bf(hsub2_bf(and_or(wh >> (4 * q), 0x000F000Fu, 0x43004300u), 0x43004300u), S1, B1);
        }
        const uint32_t a0[4] = {al[0], ah[0], al[1], ah[1]};  // k-step 2j: pairs (0,4) (1,5)
        const uint32_t a1[4] = {al[2], ah[2], al[3], ah[3]};  // k-step 2j+1: pairs (2,6) (3,7)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xst + (8 * nt + r) * DEC_XS + 16 * c + 64 * j);
          const uint32_t bx0[2] = {prmt(xv.x, xv.z, 0x5410u), prmt(xv.x, xv.z, 0x7632u)};
          const uint32_t bx1[2] = {prmt(xv.y, xv.w, 0x5410u), prmt(xv.y, xv.w, 0x7632u)};
          mma_bf16_16816(acc[nt], a0, bx0);
          mma_bf16_16816(acc[nt], a1, bx1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (aborted) break;
    const int piece = int(g - dec_range_of(blk * p.C, p.U, G));
    dec_store<NT>(p, acc, piece, row_base, warp, r, c, false);
    if (seg_end == (blk + 1) * p.C)  // this range finishes the row block: its unused planes are zero
      for (int q = piece + 1; q < p.P; ++q) dec_store<NT>(p, acc, q, row_base, warp, r, c, true);
  }
  if (lane == 0 && *abort_flag) report_timeout(nullptr);
}

// Planes of b2f_qgemm_affine_decode_partials: the most ranges covering one
// row block, for G ranges over U units of C chunks.
static int dec_planes(int64_t NB, int64_t C, int64_t G) {
  const int64_t U = NB * C;
  int P = 1;
  for (int64_t b = 0; b < NB; ++b) {
    const int64_t n = dec_range_of((b + 1) * C - 1, U, G) - dec_range_of(b * C, U, G) + 1;
    if (n > P) P = int(n);
  }
  return P;
}
static int64_t dec_grid(int64_t NB, int64_t C) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                    cudaSuccess)
      sms = 148;
  }
  return std::min<int64_t>(NB * C, int64_t(sms) * DEC_CTAS);
}

B2F_DEFINE_WAIT_CONTROLS(mma)

}  // namespace b2f

using namespace b2f;

extern "C" int b2f_gather_qgemm_affine_mma(const void* x, int64_t ldx, const int32_t* x_row_index,
                                           int64_t x_row_div, int x_plan_order, int64_t A, int64_t E,
                                           const uint32_t* w_gate, const void* s_gate, const void* b_gate,
                                           const uint32_t* w_up, const void* s_up, const void* b_up, int64_t N,
                                           int64_t K, int bits, int group_size, int tile, void* plan_workspace,
                                           int64_t plan_workspace_bytes, void* out, int64_t ldo,
                                           int out_plan_order, void* stream) {
  if (bits != 4 || group_size != 64) return B2F_ERR_UNSUPPORTED;
  if (K <= 0 || K % 128 != 0 || N <= 0 || N % 8 != 0) return B2F_ERR_UNSUPPORTED;
  if (!(tile == 16 || tile == 32 || (tile == 64 && !w_up))) return B2F_ERR_UNSUPPORTED;
  if (A < 0 || E <= 0) return B2F_ERR_INVALID;
  if (A == 0) return B2F_OK;
  if (!x || !w_gate || !s_gate || !b_gate || !out) return B2F_ERR_INVALID;
  if (w_up && (!s_up || !b_up)) return B2F_ERR_INVALID;
  if (!x_plan_order && !x_row_index && x_row_div <= 0) return B2F_ERR_INVALID;
  if (ldx < K || ldo < N) return B2F_ERR_INVALID;
  if (E * N > 0x7fffffffLL) return B2F_ERR_UNSUPPORTED;
  if (!aligned(x, 16) || ldx % 8 != 0 || !aligned(w_gate, 16) || (w_up && !aligned(w_up, 16)) || !aligned(out, 4) ||
      ldo % 2 != 0 || !aligned(s_gate, 4) || !aligned(b_gate, 4) || (w_up && (!aligned(s_up, 4) || !aligned(b_up, 4))))
    return B2F_ERR_ALIGN;
  const int64_t need = b2f_moe_plan_workspace_bytes(A, E, tile);
  if (!plan_workspace || plan_workspace_bytes < need) return B2F_ERR_WORKSPACE;
  const int64_t max_slots = b2f_moe_plan_max_slots(A, E, tile);
  if (max_slots > 0x7fffffffLL) return B2F_ERR_UNSUPPORTED;
  int rc = get_encoder();
  if (rc != B2F_OK) return rc;
  char* ws = static_cast<char*>(plan_workspace);
  MmaParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.x_row_index = x_row_index;
  p.x_row_div = x_row_div > 0 ? x_row_div : 1;
  p.s[0] = static_cast<const __nv_bfloat16*>(s_gate);
  p.b[0] = static_cast<const __nv_bfloat16*>(b_gate);
  p.s[1] = static_cast<const __nv_bfloat16*>(s_up);
  p.b[1] = static_cast<const __nv_bfloat16*>(b_up);
  p.N = N;
  p.K = K;
  p.G = int(K / 64);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.out_plan = out_plan_order ? 1 : 0;
  p.slot_count = reinterpret_cast<const int32_t*>(ws);
  p.err = reinterpret_cast<int32_t*>(ws) + 1;  // the plan header's status word
  p.slots = reinterpret_cast<const int4*>(ws + plan_slots_offset(A, E, tile));
  p.sorted = reinterpret_cast<const int32_t*>(ws + plan_sorted_offset(A, E, tile));
  p.cpk = int(K / 128);
  cudaStream_t st = as_stream(stream);
  const bool xp = x_plan_order != 0;
  if (tile == 64)
    return xp ? launch_mma_cfg<1, true, 64>(p, w_gate, nullptr, E, max_slots, 1, st)
              : launch_mma_cfg<1, false, 64>(p, w_gate, nullptr, E, max_slots, 1, st);
  if (tile == 32) {
    if (w_up)
      return xp ? launch_mma_cfg<2, true, 32>(p, w_gate, w_up, E, max_slots, 1, st)
                : launch_mma_cfg<2, false, 32>(p, w_gate, w_up, E, max_slots, 1, st);
    return xp ? launch_mma_cfg<1, true, 32>(p, w_gate, nullptr, E, max_slots, 1, st)
              : launch_mma_cfg<1, false, 32>(p, w_gate, nullptr, E, max_slots, 1, st);
  }
  if (w_up) {
    return xp ? launch_mma_cfg<2, true, 16>(p, w_gate, w_up, E, max_slots, 1, st)
              : launch_mma_cfg<2, false, 16>(p, w_gate, w_up, E, max_slots, 1, st);
  }
  return xp ? launch_mma_cfg<1, true, 16>(p, w_gate, nullptr, E, max_slots, 1, st)
            : launch_mma_cfg<1, false, 16>(p, w_gate, nullptr, E, max_slots, 1, st);
}

// rows per packed tile: the CTA rows of one matrix at plan tile 16
static int mma_packed_rows(int mat) { return mat == 2 ? MMA_CW * MmaShape<16>::WROWS / 2 : MMA_CW * MmaShape<16>::WROWS; }

extern "C" int64_t b2f_mma_packed_bytes(int64_t E, int64_t N, int64_t K, int mat) {
  if (E <= 0 || N <= 0 || K <= 0 || K % 128 != 0 || !(mat == 1 || mat == 2)) return 0;
  const int cr = mma_packed_rows(mat);
  const int64_t nb = (N + cr - 1) / cr;
  return E * nb * (K / 128) * int64_t(cr) * 72;
}

extern "C" int b2f_mma_repack(const uint32_t* wq, const void* scales, const void* biases, int64_t E, int64_t N,
                              int64_t K, int mat, void* out, int64_t out_bytes, void* stream) {
  if (E <= 0 || N <= 0 || K <= 0 || K % 128 != 0 || !(mat == 1 || mat == 2)) return B2F_ERR_INVALID;
  if (!wq || !scales || !biases || !out) return B2F_ERR_INVALID;
  if (out_bytes < b2f_mma_packed_bytes(E, N, K, mat)) return B2F_ERR_WORKSPACE;
  if (!aligned(wq, 16) || !aligned(out, 16) || !aligned(scales, 4) || !aligned(biases, 4)) return B2F_ERR_ALIGN;
  const int cr = mma_packed_rows(mat);
  const int64_t nb = (N + cr - 1) / cr;
  const int64_t groups = E * nb * (K / 128) * (cr * 4 + cr / 2);
  int64_t grid = (groups + 255) / 256;
  if (grid > 148 * 32) grid = 148 * 32;
  mma_repack_kernel<<<unsigned(grid), 256, 0, as_stream(stream)>>>(
      wq, static_cast<const uint16_t*>(scales), static_cast<const uint16_t*>(biases), E, N, K, cr, nb,
      static_cast<uint4*>(out));
  return check_launch();
}

// stream-K workspace: arrival counters for sms * CTAS CTAs (256-byte
// padded), then two 4096-float partials per CTA
static int mma_sk_ctas() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                  cudaSuccess)
    return 0;
  return sms * MmaShape<16>::CTAS;
}
static int64_t mma_sk_counter_bytes() { return (int64_t(mma_sk_ctas()) * 4 + 255) / 256 * 256; }

extern "C" int64_t b2f_mma_streamk_workspace_bytes() {
  const int64_t g = mma_sk_ctas();
  if (g <= 0) return 0;
  return mma_sk_counter_bytes() + g * 2 * 4096 * int64_t(sizeof(float));
}

extern "C" int b2f_gather_qgemm_affine_mma_packed(const void* x, int64_t ldx, const int32_t* x_row_index,
                                                  int64_t x_row_div, int x_plan_order, int64_t A, int64_t E,
                                                  const void* pw_gate, const void* pw_up, int64_t N, int64_t K,
                                                  int bits, int group_size, int tile, void* plan_workspace,
                                                  int64_t plan_workspace_bytes, void* out, int64_t ldo,
                                                  int out_plan_order, void* sk_workspace,
                                                  int64_t sk_workspace_bytes, int launch_flags, void* stream) {
  if (bits != 4 || group_size != 64 || tile != 16) return B2F_ERR_UNSUPPORTED;
  if (K <= 0 || K % 128 != 0 || N <= 0 || N % 8 != 0) return B2F_ERR_UNSUPPORTED;
  if (A < 0 || E <= 0) return B2F_ERR_INVALID;
  if (A == 0) return B2F_OK;
  if (!x || !pw_gate || !out) return B2F_ERR_INVALID;
  if (!x_plan_order && !x_row_index && x_row_div <= 0) return B2F_ERR_INVALID;
  if (ldx < K || ldo < N) return B2F_ERR_INVALID;
  if (E * N > 0x7fffffffLL) return B2F_ERR_UNSUPPORTED;
  if (!aligned(x, 16) || ldx % 8 != 0 || !aligned(pw_gate, 16) || (pw_up && !aligned(pw_up, 16)) ||
      !aligned(out, 4) || ldo % 2 != 0)
    return B2F_ERR_ALIGN;
  const int64_t need = b2f_moe_plan_workspace_bytes(A, E, tile);
  if (!plan_workspace || plan_workspace_bytes < need) return B2F_ERR_WORKSPACE;
  const int64_t max_slots = b2f_moe_plan_max_slots(A, E, tile);
  if (max_slots > 0x7fffffffLL) return B2F_ERR_UNSUPPORTED;
  char* ws = static_cast<char*>(plan_workspace);
  MmaParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.x_row_index = x_row_index;
  p.x_row_div = x_row_div > 0 ? x_row_div : 1;
  if (launch_flags & ~3) return B2F_ERR_INVALID;
  p.flags = launch_flags;
  p.pw[0] = static_cast<const uint8_t*>(pw_gate);
  p.pw[1] = static_cast<const uint8_t*>(pw_up);
  const int mat = pw_up ? 2 : 1;
  p.nb = (N + mma_packed_rows(mat) - 1) / mma_packed_rows(mat);
  p.N = N;
  p.K = K;
  p.G = int(K / 64);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.out_plan = out_plan_order ? 1 : 0;
  p.slot_count = reinterpret_cast<const int32_t*>(ws);
  p.err = reinterpret_cast<int32_t*>(ws) + 1;
  p.slots = reinterpret_cast<const int4*>(ws + plan_slots_offset(A, E, tile));
  p.sorted = reinterpret_cast<const int32_t*>(ws + plan_sorted_offset(A, E, tile));
  p.cpk = int(K / 128);
  if (sk_workspace) {
    const int64_t skb = b2f_mma_streamk_workspace_bytes();
    if (skb <= 0 || sk_workspace_bytes < skb) return B2F_ERR_WORKSPACE;
    if (!aligned(sk_workspace, 256)) return B2F_ERR_ALIGN;
    p.sk_cnt = static_cast<int32_t*>(sk_workspace);
    p.sk_part = reinterpret_cast<float*>(static_cast<char*>(sk_workspace) + mma_sk_counter_bytes());
  }
  cudaStream_t st = as_stream(stream);
  const bool xp = x_plan_order != 0;
  if (pw_up)
    return xp ? launch_mma_cfg<2, true, 16, 4, false, true>(p, nullptr, nullptr, E, max_slots, 1, st)
              : launch_mma_cfg<2, false, 16, 4, false, true>(p, nullptr, nullptr, E, max_slots, 1, st);
  return xp ? launch_mma_cfg<1, true, 16, 4, false, true>(p, nullptr, nullptr, E, max_slots, 1, st)
            : launch_mma_cfg<1, false, 16, 4, false, true>(p, nullptr, nullptr, E, max_slots, 1, st);
}

extern "C" int b2f_qgemm_decode_planes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || M > 64 || N <= 0 || K <= 0 || K % 128 != 0) return 0;
  const int64_t NB = (N + DEC_ROWS - 1) / DEC_ROWS, C = K / 128;
  return dec_planes(NB, C, dec_grid(NB, C));
}

extern "C" int b2f_qgemm_affine_decode_partials(const void* x, int64_t ldx, int64_t M, const uint32_t* wq,
                                                const void* scales, const void* biases, int64_t N, int64_t K,
                                                int bits, int group_size, float* partial, int64_t partial_bytes,
                                                void* stream) {
  if (bits != 4 || group_size != 64) return B2F_ERR_UNSUPPORTED;
  if (M < 0 || N <= 0 || K <= 0) return B2F_ERR_INVALID;
  if (M > 64 || K % 128 != 0 || N % 8 != 0 || N > 0x7fffffffLL) return B2F_ERR_UNSUPPORTED;
  if (M == 0) return B2F_OK;
  if (!x || !wq || !scales || !biases || !partial) return B2F_ERR_INVALID;
  if (ldx < K) return B2F_ERR_INVALID;
  if (!aligned(x, 16) || ldx % 8 != 0 || !aligned(wq, 16) || !aligned(partial, 8) || !aligned(scales, 4) ||
      !aligned(biases, 4))
    return B2F_ERR_ALIGN;
  const int64_t NB = (N + DEC_ROWS - 1) / DEC_ROWS, C = K / 128;
  const int64_t G = dec_grid(NB, C);
  DecParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.M = int(M);
  p.sc = static_cast<const uint32_t*>(scales);
  p.bi = static_cast<const uint32_t*>(biases);
  p.N = N;
  p.G = int(K / 64);
  p.C = int(C);
  p.U = NB * C;
  p.P = dec_planes(NB, C, G);
  p.partial = partial;
  if (partial_bytes < int64_t(p.P) * M * N * int64_t(sizeof(float))) return B2F_ERR_WORKSPACE;
  int rc = get_encoder();
  if (rc != B2F_OK) return rc;
  CUtensorMap tm{}, tmx{};
  rc = make_mma_weight_map(&tm, wq, N, K, DEC_ROWS, 4);
  if (rc != B2F_OK) return rc;
  {
    // x as bf16 [M rows, K columns]; box 160 columns x 64 rows, no swizzle
    const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(M)};
    const cuuint64_t strides[1] = {cuuint64_t(ldx) * 2};
    const cuuint32_t box[2] = {uint32_t(DEC_XS / 2), 64u};
    const cuuint32_t estr[2] = {1, 1};
    if (g_encode(&tmx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return B2F_ERR_INVALID;
  }
  const int S = DEC_STAGES;
  const int smem = S * DEC_STAGE + 1024 + 256;
  auto kern = M <= 16 ? qgemm_decode_kernel<2> : (M <= 32 ? qgemm_decode_kernel<4> : qgemm_decode_kernel<8>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return B2F_ERR_CUDA;
  }
  p.stages = S;
  return launch_kernel(kern, dim3{unsigned(G)}, dim3{unsigned(32 * (DEC_CW + 1))}, size_t(smem), as_stream(stream),
                       p, tm, tmx);
}

extern "C" int b2f_mma_splitk_ranges(int64_t K, int ksplit) {
  if (K <= 0 || K % 128 != 0) return 0;
  int cpk = 0;
  return mma_splitk_ranges(K, ksplit, &cpk);
}

extern "C" int64_t b2f_mma_splitk_workspace_bytes(int64_t A, int64_t N, int64_t K, int ksplit) {
  if (A <= 0 || N <= 0 || K <= 0 || K % 128 != 0) return 0;
  int cpk = 0;
  return int64_t(mma_splitk_ranges(K, ksplit, &cpk)) * A * N * int64_t(sizeof(float));
}

extern "C" int b2f_gather_qgemm_affine_mma_partials(const void* x, int64_t ldx, const int32_t* x_row_index,
                                                    int64_t x_row_div, int64_t A, int64_t E, const uint32_t* w,
                                                    const void* scales, const void* biases, int64_t N, int64_t K,
                                                    int bits, int group_size, int tile, void* plan_workspace,
                                                    int64_t plan_workspace_bytes, int ksplit, float* partial,
                                                    int64_t partial_bytes, void* stream) {
  if (bits != 4 || group_size != 64) return B2F_ERR_UNSUPPORTED;
  if (K <= 0 || K % 128 != 0 || N <= 0 || N % 8 != 0) return B2F_ERR_UNSUPPORTED;
  if (tile != 16 && tile != 64) return B2F_ERR_UNSUPPORTED;
  if (A < 0 || E <= 0 || ksplit < 1 || ksplit > 65535) return B2F_ERR_INVALID;
  if (A == 0) return B2F_OK;
  if (!x || !w || !scales || !biases || !partial) return B2F_ERR_INVALID;
  if (!x_row_index && x_row_div <= 0) return B2F_ERR_INVALID;
  if (ldx < K) return B2F_ERR_INVALID;
  if (E * N > 0x7fffffffLL) return B2F_ERR_UNSUPPORTED;
  if (!aligned(x, 16) || ldx % 8 != 0 || !aligned(w, 16) || !aligned(partial, 16) || !aligned(scales, 4) ||
      !aligned(biases, 4))
    return B2F_ERR_ALIGN;
  const int64_t need = b2f_moe_plan_workspace_bytes(A, E, tile);
  if (!plan_workspace || plan_workspace_bytes < need) return B2F_ERR_WORKSPACE;
  if (partial_bytes < b2f_mma_splitk_workspace_bytes(A, N, K, ksplit)) return B2F_ERR_WORKSPACE;
  const int64_t max_slots = b2f_moe_plan_max_slots(A, E, tile);
  if (max_slots > 65535) return B2F_ERR_UNSUPPORTED;
  int rc = get_encoder();
  if (rc != B2F_OK) return rc;
  char* ws = static_cast<char*>(plan_workspace);
  MmaParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.x_row_index = x_row_index;
  p.x_row_div = x_row_div > 0 ? x_row_div : 1;
  p.s[0] = p.s[1] = static_cast<const __nv_bfloat16*>(scales);
  p.b[0] = p.b[1] = static_cast<const __nv_bfloat16*>(biases);
  p.N = N;
  p.K = K;
  p.G = int(K / 64);
  p.ldo = N;
  p.slot_count = reinterpret_cast<const int32_t*>(ws);
  p.err = reinterpret_cast<int32_t*>(ws) + 1;
  p.slots = reinterpret_cast<const int4*>(ws + plan_slots_offset(A, E, tile));
  p.sorted = reinterpret_cast<const int32_t*>(ws + plan_sorted_offset(A, E, tile));
  const int ks = mma_splitk_ranges(K, ksplit, &p.cpk);
  p.partial = partial;
  p.plane = A * N;
  // 64-token tiles: one unpack of each weight serves a whole decode batch
  if (tile == 64) return launch_mma_cfg<1, false, 64>(p, w, nullptr, E, max_slots, ks, as_stream(stream));
  return launch_mma_cfg<1, false, 16>(p, w, nullptr, E, max_slots, ks, as_stream(stream));
}

extern "C" int b2f_gather_qgemm_2bit_mma(const void* x, int64_t ldx, const int32_t* x_row_index, int64_t x_row_div,
                                         int64_t A, int64_t E, const uint32_t* w_gate, const void* s_gate,
                                         const void* b_gate, const uint32_t* w_up, const void* s_up,
                                         const void* b_up, int64_t N, int64_t K, int scale_dtype, int tile,
                                         void* plan_workspace, int64_t plan_workspace_bytes, void* out, int64_t ldo,
                                         void* stream) {
  if (!(scale_dtype == B2F_BF16 || scale_dtype == B2F_F16)) return B2F_ERR_UNSUPPORTED;
  if (K <= 0 || K % 128 != 0 || N <= 0 || N % 8 != 0 || tile != 16) return B2F_ERR_UNSUPPORTED;
  if (A < 0 || E <= 0) return B2F_ERR_INVALID;
  if (A == 0) return B2F_OK;
  if (!x || !w_gate || !s_gate || !b_gate || !out) return B2F_ERR_INVALID;
  if (w_up && (!s_up || !b_up)) return B2F_ERR_INVALID;
  if (!x_row_index && x_row_div <= 0) return B2F_ERR_INVALID;
  if (ldx < K || ldo < N) return B2F_ERR_INVALID;
  if (E * N > 0x7fffffffLL) return B2F_ERR_UNSUPPORTED;
  if (!aligned(x, 16) || ldx % 8 != 0 || !aligned(w_gate, 16) || (w_up && !aligned(w_up, 16)) || !aligned(out, 4) ||
      ldo % 2 != 0 || !aligned(s_gate, 4) || !aligned(b_gate, 4) || (w_up && (!aligned(s_up, 4) || !aligned(b_up, 4))))
    return B2F_ERR_ALIGN;
  const int64_t need = b2f_moe_plan_workspace_bytes(A, E, tile);
  if (!plan_workspace || plan_workspace_bytes < need) return B2F_ERR_WORKSPACE;
  const int64_t max_slots = b2f_moe_plan_max_slots(A, E, tile);
  if (max_slots > 65535) return B2F_ERR_UNSUPPORTED;
  int rc = get_encoder();
  if (rc != B2F_OK) return rc;
  char* ws = static_cast<char*>(plan_workspace);
  MmaParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.x_row_index = x_row_index;
  p.x_row_div = x_row_div > 0 ? x_row_div : 1;
  p.s[0] = static_cast<const __nv_bfloat16*>(s_gate);
  p.b[0] = static_cast<const __nv_bfloat16*>(b_gate);
  p.s[1] = static_cast<const __nv_bfloat16*>(s_up);
  p.b[1] = static_cast<const __nv_bfloat16*>(b_up);
  p.N = N;
  p.K = K;
  p.G = int(K / 64);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.slot_count = reinterpret_cast<const int32_t*>(ws);
  p.err = reinterpret_cast<int32_t*>(ws) + 1;
  p.slots = reinterpret_cast<const int4*>(ws + plan_slots_offset(A, E, tile));
  p.sorted = reinterpret_cast<const int32_t*>(ws + plan_sorted_offset(A, E, tile));
  p.cpk = int(K / 128);
  cudaStream_t st = as_stream(stream);
  const bool f16 = scale_dtype == B2F_F16;
  if (w_up)
    return f16 ? launch_mma_cfg<2, false, 16, 2, true>(p, w_gate, w_up, E, max_slots, 1, st)
               : launch_mma_cfg<2, false, 16, 2, false>(p, w_gate, w_up, E, max_slots, 1, st);
  return f16 ? launch_mma_cfg<1, false, 16, 2, true>(p, w_gate, nullptr, E, max_slots, 1, st)
             : launch_mma_cfg<1, false, 16, 2, false>(p, w_gate, nullptr, E, max_slots, 1, st);
}
