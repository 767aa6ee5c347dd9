/*
 * b2f.h -- C ABI of libb200flash.so, the B200 (sm_100a) kernels behind
 * MLX-Flash's quantized-weight / quantized-KV-cache hot path.
 *
 * Conventions (every entry point):
 *   - plain device pointers, int64 sizes, and an opaque `stream`
 *     (a cudaStream_t passed as void*; NULL means the legacy default stream);
 *   - returns an int status: B2F_OK (0) or a negative B2F_ERR_* code; a CUDA
 *     launch error is reported as B2F_ERR_CUDA and its cudaError_t text is
 *     available from b2f_last_error_string();
 *   - the library never allocates: outputs and workspaces are owned by the
 *     caller (the Python layer allocates them as torch tensors);
 *   - entry points are stream-ordered and hold no global mutable state (the
 *     launch policy of b2f_set_launch_pdl is per thread), so different
 *     threads may drive different streams concurrently.
 *
 * Data formats:
 *   AFFINE (weights): W[rows, K] -> wq uint32[rows, K*bits/32] packed
 *     least-significant field first (element k at bit bits*(k%(32/bits)) of
 *     word k/(32/bits)); scales/biases [rows, K/group_size] in the weight dtype;
 *     w = q*scale + bias.
 *   KV-SYM (reference KV format, quantized_kv_cache.py:68-234): per row of D
 *     values, groups of gs=min(group_size,D); scale=absmax/(2^(bits-1)-1) in
 *     float32; codes offset by max_int into uint8; 4-bit byte = c[2i]<<4|c[2i+1];
 *     2-bit byte = c0<<6|c1<<4|c2<<2|c3.
 */
#ifndef B2F_H_
#define B2F_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define B2F_OK 0
#define B2F_ERR_INVALID (-1)      /* bad pointer / shape / stride argument */
#define B2F_ERR_UNSUPPORTED (-2)  /* bits / group_size / dtype / size not supported */
#define B2F_ERR_ALIGN (-3)        /* pointer or stride alignment violated */
#define B2F_ERR_CUDA (-4)         /* CUDA launch/runtime error */
#define B2F_ERR_TIMEOUT (-5)      /* a bounded device wait gave up */
#define B2F_ERR_WORKSPACE (-6)    /* workspace missing or too small */

/* element dtypes */
#define B2F_BF16 0
#define B2F_F16 1
#define B2F_F32 2

/* ---- library info --------------------------------------------------- */
const char* b2f_version(void);
const char* b2f_status_string(int status);
/* text of the last CUDA error seen by this thread (or "") */
const char* b2f_last_error_string(void);

/* Bounded device waits.  Every kernel that waits on a copy or on another warp
 * (the expert GEMMs, the GEMV, the paged decode attention) gives up after a
 * time limit instead of spinning forever, skips its remaining work and
 * records B2F_ERR_TIMEOUT in its call's status word (the MoE plan header, for
 * the plan-driven GEMMs) and in a library-wide sticky status.
 * b2f_device_status synchronises the device and reads that sticky status
 * (B2F_OK or B2F_ERR_TIMEOUT) into *status_out, clearing it if `clear`. */
int b2f_device_status(int32_t* status_out, int clear);

/* The wait limit in ns for all later launches (0: the default, 2 s). */
int b2f_set_wait_limit_ns(int64_t ns);

/* Test control: non-zero makes the kernels' producer warps issue no copies,
 * so their consumers' bounded waits run out (how the tests drive the timeout
 * path without any fault); 0 (the default) is normal operation. */
int b2f_set_producer_stall(int on);

/* Launch policy of the calling thread (default 0).  Non-zero: the decode-step
 * kernels are launched as programmatic dependent launches, so each may be
 * scheduled while the kernel before it in the stream runs its last wave; each
 * waits for that kernel's completion before touching memory and only then
 * lets the next one be scheduled.  Results are identical either way; a CUDA
 * graph captured under the policy keeps it.  Returns the previous value. */
int b2f_set_launch_pdl(int on);

/* ---- (a) affine quantize / (a') dequantize ---------------------------- */

/* mx.quantize(w, group_size, bits) as called through
 * nn.QuantizedLinear.from_linear (mlx_flash_compress/layer_quantization.py:254)
 * and nn.quantize (mlx_flash_compress/dflash_model.py:300), with MLX's
 * per-group rule: scale = max((max-min)/(2^bits-1), 1e-7), the edge (the
 * larger-magnitude end) becomes the bias and an exact code (scale = edge/q0,
 * negative when the edge is the max), q from the f32 scale and bias.
 * w: [rows, K] of `dtype`; wq: uint32 [rows, K*bits/32]; scales, biases:
 * [rows, K/group_size] of `dtype`.  bits in {2,4,8}; group_size in {32,64,128}. */
int b2f_quantize_affine(const void* w, int dtype, int64_t rows, int64_t K, int bits,
                        int group_size, uint32_t* wq, void* scales, void* biases,
                        void* stream);

/* The same packing with the min/max rule: scale = (max-min)/(2^bits-1)
 * rounded to `dtype`, bias = min, q from the rounded scale (q = 0 where it is
 * 0).  No MLX call corresponds to it; it is the rule stated for the
 * single-linear workload (W[4096,4096], 4-bit, group 64). */
int b2f_quantize_affine_minmax(const void* w, int dtype, int64_t rows, int64_t K, int bits,
                               int group_size, uint32_t* wq, void* scales, void* biases,
                               void* stream);

/* mx.dequantize (the unpack restated at mlx_flash_compress/mixed_precision.py:150-171).
 * If row_index is non-NULL, output row i is source row row_index[i] (an
 * embedding-style gather); otherwise out_rows must equal the source rows. */
int b2f_dequantize_affine(const uint32_t* wq, const void* scales, const void* biases,
                          int dtype, int64_t out_rows, int64_t K, int bits,
                          int group_size, const int32_t* row_index, void* out,
                          void* stream);

/* ---- (b) dequant-GEMV, dense ----------------------------------------- */

/* mx.quantized_matmul(x, wq, scales, biases, transpose=True, group_size, bits),
 * the forward of nn.QuantizedLinear swapped in at layer_quantization.py:254.
 * x bf16 [M, K] (row stride ldx elements); wq [N, K*bits/32]; scales/biases
 * bf16 [N, K/group_size]; y bf16 [M, N] (row stride ldy).  If residual is
 * non-NULL (bf16 [M, N], stride ldy) y = residual + x.W^T.
 * bits in {4,8}; group_size in {32,64,128}; K % group_size == 0; K <= 64*group_size. */
int b2f_qgemv_affine(const void* x, int64_t ldx, int64_t M, const uint32_t* wq,
                     const void* scales, const void* biases, int64_t N, int64_t K,
                     int bits, int group_size, const void* residual, void* y,
                     int64_t ldy, void* stream);

/* ---- (b) grouped dequant-GEMV (routed experts) ------------------------ */

/* Workspace bytes needed by b2f_moe_plan for A assignments over E experts
 * with token tiles of `tile` rows. */
int64_t b2f_moe_plan_workspace_bytes(int64_t A, int64_t E, int tile);

/* Upper bound on the number of (expert, token-tile) slots the plan can emit. */
int64_t b2f_moe_plan_max_slots(int64_t A, int64_t E, int tile);

/* Groups the A assignments by expert (counting sort on the GPU) and cuts each
 * expert's list into tiles of at most `tile` assignments.  expert_of[a] is the
 * expert of assignment a (the rhs_indices of mx.gather_qmm at
 * expert_streaming.py:230-241, after the lookup remap at :228).  The plan lives
 * in `workspace` (b2f_moe_plan_workspace_bytes) and is consumed by
 * b2f_gather_qgemv_affine.  Out-of-range expert ids make the call fail with
 * B2F_ERR_INVALID reported through `status_out` (device int32, may be NULL). */
int b2f_moe_plan(const int32_t* expert_of, int64_t A, int64_t E, int tile,
                 void* workspace, int64_t workspace_bytes, int32_t* status_out,
                 void* stream);

/* mx.gather_qmm(x, w, scales, biases, rhs_indices=..., transpose=True,
 * group_size, bits) -- expert_streaming.py:230-241.
 * For every assignment a: out[a, :] = x[x_row[a], :] . W[expert_of[a]]^T,
 * where x_row[a] = x_row_index ? x_row_index[a] : a / x_row_div.
 * w_gate: stacked [E, N, K*bits/32] (+ scales/biases [E, N, K/gs]).
 * If w_up is non-NULL the call computes the SwitchGLU front half instead:
 * out[a, :] = silu(x.Wgate^T) * (x.Wup^T)  (kernels/ops.py:48-108 fused in).
 * The plan must come from b2f_moe_plan with the same expert_of and `tile`. */
int b2f_gather_qgemv_affine(const void* x, int64_t ldx, const int32_t* x_row_index,
                            int64_t x_row_div, int64_t A, int64_t E,
                            const uint32_t* w_gate, const void* s_gate, const void* b_gate,
                            const uint32_t* w_up, const void* s_up, const void* b_up,
                            int64_t N, int64_t K, int bits, int group_size, int tile,
                            const void* plan_workspace, int64_t plan_workspace_bytes,
                            void* out, int64_t ldo, void* stream);

/* ---- (c) tcgen05/TMEM grouped GEMM (prefill and large decode tiles) ----- */

/* Same contract as b2f_qgemv_affine, computed on the 5th-generation tensor
 * cores: 128 weight rows x `tile` tokens per CTA (tile a multiple of 16,
 * <= 256), weights dequantized to bf16 in shared memory, fp32 accumulators in
 * tensor memory.  group_size must be 64; bits in {4,8}; K % 64 == 0.  This is
 * mx.quantized_matmul for many tokens (prefill of QuantizedLinear,
 * layer_quantization.py:254). */
int b2f_qgemm_affine_tcgen05(const void* x, int64_t ldx, int64_t M, const uint32_t* wq,
                             const void* scales, const void* biases, int64_t N, int64_t K,
                             int bits, int group_size, const void* residual, void* y,
                             int64_t ldy, int tile, void* stream);

/* mx.gather_qmm on the tensor cores (expert_streaming.py:230-241 at prefill
 * sizes): same arguments and plan as b2f_gather_qgemv_affine, with the plan
 * built by b2f_moe_plan for the same `tile` (16..256, multiple of 16). */
int b2f_gather_qgemm_affine_tcgen05(const void* x, int64_t ldx, const int32_t* x_row_index,
                                    int64_t x_row_div, int64_t A, int64_t E,
                                    const uint32_t* w_gate, const void* s_gate,
                                    const void* b_gate, const uint32_t* w_up, const void* s_up,
                                    const void* b_up, int64_t N, int64_t K, int bits,
                                    int group_size, int tile, const void* plan_workspace,
                                    int64_t plan_workspace_bytes, void* out, int64_t ldo,
                                    void* stream);

/* ---- (a-kv) reference KV quantizer ------------------------------------ */

/* Packed bytes per row and groups per row for a last axis of length D. */
int64_t b2f_kv_packed_len(int64_t D, int bits, int group_size);
int64_t b2f_kv_num_groups(int64_t D, int group_size);

/* quantize_tensor(x, bits, group_size) -- quantized_kv_cache.py:68-156.
 * x: [rows, D] of `dtype` (bf16/f16/f32: arithmetic follows the dtype, like
 * MLX does).  Row r is written to packed row dst_row[r] (or r if dst_row is
 * NULL) of `packed` (row stride packed_ld bytes) and scales row dst_row[r]
 * (stride scales_ld floats); zeros (same layout as scales) may be NULL. */
int b2f_kv_quantize_sym(const void* x, int dtype, int64_t rows, int64_t D, int bits,
                        int group_size, const int64_t* dst_row, uint8_t* packed,
                        int64_t packed_ld, float* scales, float* zeros,
                        int64_t scales_ld, void* stream);

/* dequantize_tensor(...) -- quantized_kv_cache.py:159-234; float32 output
 * [rows, D].  Row r is read from src_row[r] (or r) of packed/scales. */
int b2f_kv_dequantize_sym(const uint8_t* packed, int64_t packed_ld, const float* scales,
                          int64_t scales_ld, const int64_t* src_row, int64_t rows,
                          int64_t D, int bits, int group_size, float* out, void* stream);

/* ---- (d) paged decode attention over packed K/V ----------------------- */

/* Workspace bytes for b2f_qkv_decode_attn with the given split count. */
int64_t b2f_qkv_decode_attn_workspace_bytes(int64_t B, int64_t Hq, int64_t D, int n_splits);

/* Decode attention for 1 query token per sequence over a paged KV cache in
 * the reference KV format (the fp32 SDPA the caller of
 * quantized_kv_cache.py:311-358 performs, without materialising fp32 K/V).
 * q: bf16 [B, Hq, D]; out: bf16 [B, Hq, D].
 * A page holds Hkv*page_size rows of packed_len(D) code bytes (and D/64 f32
 * scales); the row of (head h, slot s) in page P is
 *   P*Hkv*page_size + h*head_stride + s*slot_stride,
 * head-major pages: head_stride=page_size, slot_stride=1
 * token-major pages (the reference's [S, H, D] chunk order): head_stride=1,
 * slot_stride=Hkv.
 * block_table: int32 [B, max_pages]; seq_lens: int32 [B].
 * Hq % Hkv == 0, Hq/Hkv <= 16; D in {64,128,256}; bits in {2,4,8}; gs=64 (or D
 * if D<64); page_size % 16 == 0.  n_splits >= 1 splits each sequence. */
int b2f_qkv_decode_attn(const void* q, const uint8_t* k_pages, const float* k_scales,
                        const uint8_t* v_pages, const float* v_scales,
                        const int32_t* block_table, int64_t max_pages,
                        const int32_t* seq_lens, int64_t B, int64_t Hq, int64_t Hkv,
                        int64_t D, int64_t page_size, int64_t head_stride,
                        int64_t slot_stride, int bits, int group_size,
                        float softmax_scale, int n_splits, void* workspace,
                        int64_t workspace_bytes, void* out, void* stream);

/* Allocation-free form of b2f_qkv_decode_attn (no counterpart in the
 * reference): the split-K partial results go to a fixed device array inside
 * the library instead of a caller workspace, for callers that cannot allocate
 * device memory (a C/cgo/JNI host without a device allocator, a process whose
 * GPU memory is owned by another framework's pool, or a path where a
 * synchronising cudaMalloc is not acceptable).
 *   - capacity: B2F_ATTN_NOALLOC_SCRATCH_BYTES; a call whose workspace
 *     (b2f_qkv_decode_attn_workspace_bytes) would exceed it returns
 *     B2F_ERR_WORKSPACE without launching anything;
 *   - the array is part of the loaded library: every GPU that loads it holds
 *     4 MiB until the process exits;
 *   - the first call on a device (that device must be current) looks up the
 *     array's device address with cudaGetSymbolAddress and caches it; make that
 *     first call before any stream capture;
 *   - all calls on a device share the array and it keeps the last call's
 *     contents (nothing needs clearing: every byte read is written first);
 *     calls that overlap on the GPU race on it, so serialise them.
 * Arguments and results are those of b2f_qkv_decode_attn without the
 * workspace pair.  It allocates nothing. */
#define B2F_ATTN_NOALLOC_SCRATCH_BYTES (4 << 20)
int b2f_qkv_decode_attn_noalloc(const void* q, const uint8_t* k_pages, const float* k_scales,
                                const uint8_t* v_pages, const float* v_scales,
                                const int32_t* block_table, int64_t max_pages,
                                const int32_t* seq_lens, int64_t B, int64_t Hq, int64_t Hkv,
                                int64_t D, int64_t page_size, int64_t head_stride,
                                int64_t slot_stride, int bits, int group_size,
                                float softmax_scale, int n_splits, void* out, void* stream);

/* Workspace bytes of b2f_qgemm_affine_tcgen05_splitk (fp32 partials). */
int64_t b2f_qgemm_splitk_workspace_bytes(int64_t M, int64_t N, int ksplit);

/* Number of non-empty K ranges the split-K entry points use for `ksplit`
 * (ranges of ceil((K/64)/ksplit) 64-wide chunks); 0 for invalid K. */
int b2f_qgemm_splitk_ranges(int64_t K, int ksplit);

/* The first half of b2f_qgemm_affine_tcgen05_splitk: fp32 partials
 * partial[r][M][N] for r < b2f_qgemm_splitk_ranges(K, ksplit), to be summed
 * by the consumer (b2f_combine_rmsnorm_partials,
 * b2f_qk_norm_rope_kv_append_partials) instead of a separate pass. */
int b2f_qgemm_affine_tcgen05_partials(const void* x, int64_t ldx, int64_t M, const uint32_t* wq,
                                      const void* scales, const void* biases, int64_t N, int64_t K,
                                      int bits, int group_size, int tile, int ksplit, float* partial,
                                      int64_t partial_bytes, void* stream);

/* b2f_qgemm_affine_tcgen05 with K cut into `ksplit` ranges so that few
 * 128-row blocks (decode-sized M, e.g. the q/k/v and o projections at 64
 * tokens) still fill every SM: each range writes fp32 partials into
 * `workspace`, a second kernel sums them (+ residual) into bf16 y.
 * ksplit 1..64; ksplit == 1 is b2f_qgemm_affine_tcgen05. */
int b2f_qgemm_affine_tcgen05_splitk(const void* x, int64_t ldx, int64_t M, const uint32_t* wq,
                                    const void* scales, const void* biases, int64_t N, int64_t K,
                                    int bits, int group_size, const void* residual, void* y,
                                    int64_t ldy, int tile, int ksplit, void* workspace,
                                    int64_t workspace_bytes, void* stream);

/* b2f_moe_route_topk followed by b2f_moe_plan on its ids, in two launches
 * (router logits; then top-k per token with the counting sort run by the
 * last thread block to finish): expert_streaming.py:439-472 routing plus the
 * sort-by-expert of gather_qmm(sorted_indices=True).  Same outputs as the
 * two calls; plan workspace as for b2f_moe_plan(A = T*k, E, tile).  H <= 8192. */
int b2f_moe_route_plan(const void* x, int64_t T, int64_t H, const void* wr, const float* bias,
                       int64_t E, int64_t k, int renorm, float* logits_ws, int32_t* inds,
                       float* scores, int tile, void* plan_workspace, int64_t plan_workspace_bytes,
                       int32_t* status_out, void* stream);

/* ---- (c) grouped GEMM for decode-sized expert tiles (register dequant) -- */

/* mx.gather_qmm (expert_streaming.py:230-241; SwitchGLU front half of
 * kernels/ops.py:48-108 fused when w_up is non-NULL) for decode-sized expert
 * tiles: the 4-bit codes are TMA-staged in shared memory, unpacked in
 * registers and fed to warp-level tensor-core MMA (mma.sync m16n8k16 bf16,
 * 16 weight rows x 8 tokens), each 64-wide group folded as
 * s*sum(q x) + b*sum(x) in fp32 (the order MLX's quantized kernels use).
 * Plan from b2f_moe_plan / b2f_moe_route_plan / b2f_ep_plan with tile = 16
 * or 32 (expert tiles; 32 unpacks an expert routed 17-32 tokens once instead
 * of twice), or tile = 64 without w_up (wide tiles: a dense projection
 * of up to 64 decode tokens is b2f_moe_plan over all-zero expert ids, E = 1);
 * same weight format as b2f_gather_qgemm_affine_tcgen05; bits 4,
 * group_size 64, K % 128 == 0, N % 8 == 0.
 * x_plan_order = 0: x row of assignment a is x_row_index[a] (or a/x_row_div),
 *   natural column order.
 * x_plan_order = 1: x row i belongs to sorted position i of the plan and each
 *   group of 8 columns is stored in the order (0,4,1,5,2,6,3,7) (what
 *   b2f_moe_gather_rows writes, or this call with out_plan_order = 1).
 * out_plan_order = 0: out[a, :] for assignment a, natural column order.
 * out_plan_order = 1: out row i = sorted position i, columns permuted as above
 *   (the input of the down projection with x_plan_order = 1).
 * A device wait that gives up records B2F_ERR_TIMEOUT in the plan's status
 * word (int32 at byte 4 of the plan workspace). */
int b2f_gather_qgemm_affine_mma(const void* x, int64_t ldx, const int32_t* x_row_index,
                                int64_t x_row_div, int x_plan_order, int64_t A, int64_t E,
                                const uint32_t* w_gate, const void* s_gate, const void* b_gate,
                                const uint32_t* w_up, const void* s_up, const void* b_up,
                                int64_t N, int64_t K, int bits, int group_size, int tile,
                                void* plan_workspace, int64_t plan_workspace_bytes, void* out,
                                int64_t ldo, int out_plan_order, void* stream);

/* Packed expert weights for b2f_gather_qgemm_affine_mma_packed: the 4-bit
 * codes of E stacked [N, K] matrices (MLX layout, uint32 [E*N, K/8]) and
 * their bf16 scales / biases [E*N, K/64], re-laid as one tile per (expert,
 * block of 128 rows for a gate/up matrix (mat 2) or 256 rows for a down
 * matrix (mat 1), 128-wide K chunk).  A tile is the exact shared-memory
 * image the GEMM consumes: the codes (64-byte rows, 16-byte word groups
 * XOR-swizzled by (row / 2) % 4), then per row 8 bytes of scale and bias for
 * the chunk's two groups; rows past N zero-filled.  No MLX call corresponds:
 * an internal layout of HBM-resident experts, so each staged tile is one
 * contiguous bulk copy and no scale is fetched from global memory in the
 * inner loop.  out must hold b2f_mma_packed_bytes (72 bytes per row and
 * 128-wide chunk). */
int64_t b2f_mma_packed_bytes(int64_t E, int64_t N, int64_t K, int mat);
int b2f_mma_repack(const uint32_t* wq, const void* scales, const void* biases, int64_t E, int64_t N,
                   int64_t K, int mat, void* out, int64_t out_bytes, void* stream);

/* b2f_gather_qgemm_affine_mma (plan tile 16) reading b2f_mma_repack tiles
 * (mat 2 for pw_gate / pw_up with SwiGLU fused, mat 1 for pw_gate alone)
 * instead of the MLX-layout codes, scales and biases.  Same results, bit
 * for bit, as the unpacked call when sk_workspace is null.
 *
 * sk_workspace (optional, 256-byte aligned, b2f_mma_streamk_workspace_bytes
 * long): stream-K scheduling.  The live (slot, 128/256-row block) items
 * times their 128-wide K chunks are cut into one equal range per resident
 * CTA, so every SM streams the same number of weight tiles; an item cut
 * between two CTAs is summed in fp32 by the second to finish (results
 * deterministic, within fp32 rounding of the whole-item sum).  Layout: one
 * int32 arrival counter per resident CTA (SMs x 3, padded to 256 bytes),
 * then two 4096-float partials per CTA.  The counters must be ZERO before
 * the first use; each launch that completes leaves them zero (after a
 * B2F_ERR_TIMEOUT zero them again).  One workspace serves calls in stream
 * order.
 *
 * launch_flags (programmatic dependent launch; 0 = ordinary stream order):
 * bit 0 -- this call may start while the previous kernel in the stream
 * finishes: it stages its first weight tiles, then waits for that kernel
 * before copying x (so x may be that kernel's output, but the plan must be
 * older); bit 1 -- let the next kernel start once every CTA of this one has
 * passed that wait (pair it with bit 0 on the next call). */
int64_t b2f_mma_streamk_workspace_bytes(void);
int b2f_gather_qgemm_affine_mma_packed(const void* x, int64_t ldx, const int32_t* x_row_index,
                                       int64_t x_row_div, int x_plan_order, int64_t A, int64_t E,
                                       const void* pw_gate, const void* pw_up, int64_t N, int64_t K,
                                       int bits, int group_size, int tile, void* plan_workspace,
                                       int64_t plan_workspace_bytes, void* out, int64_t ldo,
                                       int out_plan_order, void* sk_workspace, int64_t sk_workspace_bytes,
                                       int launch_flags, void* stream);

/* Dense projection of a decode batch (the QuantizedLinear forward of
 * layer_quantization.py:240-256 for M <= 64 token rows: the q/k/v and o
 * projections of a decode step): fp32 planes partial[P][M][N] whose sum in
 * plane order is x . dequant(W)^T, P = b2f_qgemm_decode_planes(M, N, K)
 * (0 for unsupported sizes).  The (128-row block, 128-wide K chunk) units
 * are cut into equal contiguous ranges, one per SM (stream-K), so every SM
 * streams the same weight bytes; weights are dequantized to bf16 in
 * registers (one rounding of q*s + b, as the tcgen05 kernels) and multiplied
 * on warp MMA.  4-bit, group 64, K % 128 == 0, N % 8 == 0; x bf16 16-byte
 * aligned with ldx % 8 == 0; partial 8-byte aligned, at least P*M*N floats.
 * Consumers: b2f_qk_norm_rope_kv_append_partials, b2f_combine_rmsnorm_partials
 * with nsplit = P. */
int b2f_qgemm_decode_planes(int64_t M, int64_t N, int64_t K);
int b2f_qgemm_affine_decode_partials(const void* x, int64_t ldx, int64_t M, const uint32_t* wq,
                                     const void* scales, const void* biases, int64_t N, int64_t K, int bits,
                                     int group_size, float* partial, int64_t partial_bytes, void* stream);

/* b2f_gather_qgemm_affine_mma (tile 16, or 64: slots of up to 64 tokens,
 * one unpack of each weight for a whole decode batch; one matrix, x rows
 * x_row(a)) with K cut into ksplit ranges of whole 128-wide chunks (grid z):
 * range z writes
 * fp32 planes partial[z][a][0:N] for every planned assignment a, to be summed
 * by the consumer (b2f_qk_norm_rope_kv_append_partials,
 * b2f_combine_rmsnorm_partials).  A dense projection of B decode tokens is
 * the plan of b2f_moe_plan over B all-zero expert ids with E = 1.  The plane
 * count is b2f_mma_splitk_ranges(K, ksplit); partial 16-byte aligned, at
 * least b2f_mma_splitk_workspace_bytes(A, N, K, ksplit) bytes. */
int b2f_mma_splitk_ranges(int64_t K, int ksplit);
int64_t b2f_mma_splitk_workspace_bytes(int64_t A, int64_t N, int64_t K, int ksplit);
int b2f_gather_qgemm_affine_mma_partials(const void* x, int64_t ldx, const int32_t* x_row_index,
                                         int64_t x_row_div, int64_t A, int64_t E, const uint32_t* w,
                                         const void* scales, const void* biases, int64_t N, int64_t K,
                                         int bits, int group_size, int tile, void* plan_workspace,
                                         int64_t plan_workspace_bytes, int ksplit, float* partial,
                                         int64_t partial_bytes, void* stream);

/* b2f_gather_qgemm_affine_mma for 2-bit codes: w uint32 [E, N, K/16], code k
 * at bits 2*(k % 16) of word k/16 (LSB first: the byte layout of
 * requantize_4bit_to_2bit's packed output, mixed_precision.py:173-216, and
 * of MLX's 2-bit affine format), scales/biases [E, N, K/64] of scale_dtype
 * (B2F_F16 as requantize_4bit_to_2bit writes them, or B2F_BF16);
 * w = q*s + b, folded per group as s*sum(q x) + b*sum(x).  x rows x_row(a),
 * natural column order; out[a, :] natural; plan tile 16; SwiGLU fused when
 * w_up is given.  K % 128 == 0, N % 8 == 0. */
int b2f_gather_qgemm_2bit_mma(const void* x, int64_t ldx, const int32_t* x_row_index, int64_t x_row_div,
                              int64_t A, int64_t E, const uint32_t* w_gate, const void* s_gate,
                              const void* b_gate, const uint32_t* w_up, const void* s_up,
                              const void* b_up, int64_t N, int64_t K, int scale_dtype, int tile,
                              void* plan_workspace, int64_t plan_workspace_bytes, void* out, int64_t ldo,
                              void* stream);

/* ---- (c) grouped GEMM over expert-sorted rows (decode and prefill) ------ */

/* Copies the planned assignments' activation rows into plan order:
 * out[i, :] = x[x_row(sorted[i]), :] for i < (planned count), x_row(a) =
 * x_row_index ? x_row_index[a] : a / x_row_div, with every group of 8
 * columns stored in the order (0,4,1,5,2,6,3,7).  The plan (b2f_moe_plan or
 * b2f_ep_plan) must use the same A, E and tile.  Rows >= the planned count
 * are not written.  bf16 x [*, ldx], out [A, ldo]; K % 8 == 0. */
int b2f_moe_gather_rows(const void* x, int64_t ldx, const int32_t* x_row_index, int64_t x_row_div,
                        int64_t A, int64_t E, int tile, const void* plan_workspace,
                        int64_t plan_workspace_bytes, int64_t K, void* out, int64_t ldo,
                        void* stream);

/* mx.gather_qmm over expert-sorted rows (expert_streaming.py:224-241 with
 * sorted_indices=True) on tcgen05/TMEM: persistent CTAs walk the plan's
 * (slot, 128-row block) units; x tiles arrive by TMA from x_sorted (the
 * layout b2f_moe_gather_rows writes: plan order, permuted column groups).
 * w_up non-NULL fuses silu(x.Wg^T) * (x.Wu^T).  out_sorted = 0: out[a, n] for
 * assignment a, natural columns (the layout of b2f_gather_qgemm_affine_*);
 * out_sorted = 1: out[i, perm(n)] in plan order -- the x_sorted layout of a
 * following call (N % 8 == 0).  group_size 64, bits 4 or 8, K % 128 == 0. */
int b2f_sorted_qgemm_affine_tcgen05(const void* x_sorted, int64_t ldx, int64_t A, int64_t E,
                                    const uint32_t* w_gate, const void* s_gate, const void* b_gate,
                                    const uint32_t* w_up, const void* s_up, const void* b_up,
                                    int64_t N, int64_t K, int bits, int group_size, int tile,
                                    const void* plan_workspace, int64_t plan_workspace_bytes,
                                    void* out, int64_t ldo, int out_sorted, void* stream);

/* ---- KV eviction: attention-guided (H2O / ScissorHands) and sink + window - */

/* kv_compression.py:84-141 record_attention: per-token importance = mean over
 * the H heads of one attention row.  attn points at head 0's row; head h's
 * row starts head_stride elements later (head_stride = S_q * S for the last
 * query row of an [H, S_q, S] tensor).  mode 0: out[s] = v; 1: out[s] += v
 * (H2O accumulation); 2: out[s] = decay*out[s] + (1-decay)*v (ScissorHands
 * EMA).  out2 (may be NULL): out2[s] += v (H2O cross-layer total).  fp32
 * outputs; attn in `dtype`. */
int b2f_attn_row_head_mean(const void* attn, int dtype, int64_t H, int64_t head_stride, int64_t S,
                           int mode, float decay, float* out, float* out2, void* stream);

/* Workspace bytes of b2f_qkv_head_mean_probs. */
int64_t b2f_qkv_head_mean_probs_workspace_bytes(int64_t B, int64_t Hq, int n_splits);

/* The same importance on the paged quantized decode path (no attention
 * matrix is formed): for every sequence b and token t < seq_lens[b],
 * v = mean over the Hq query heads of softmax_t(scale * q[b,h] . K[b,t]),
 * K dequantized from the reference KV format pages exactly as
 * b2f_qkv_decode_attn reads them (same page/stride arguments); written to
 * out[b*out_ld + t] by `mode` as in b2f_attn_row_head_mean.  max_len >= every
 * seq_len; Hq/Hkv <= 16; D % 64 == 0, D <= 256. */
int b2f_qkv_head_mean_probs(const void* q, const uint8_t* k_pages, const float* k_scales,
                            const int32_t* block_table, int64_t max_pages, const int32_t* seq_lens,
                            int64_t max_len, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                            int64_t page_size, int64_t head_stride, int64_t slot_stride, int bits,
                            int group_size, float softmax_scale, int n_splits, void* workspace,
                            int64_t workspace_bytes, float* out, int64_t out_ld, int mode,
                            float decay, void* stream);

/* kv_compression.py:293-364 _compress_layer keep list for one layer of S
 * tokens: if S > budget and the middle [sink, S-window) holds more than
 * budget - sink - window tokens, keep = sink tokens, the most important
 * middle tokens (importance[t] descending, ties to the lower position;
 * importance NULL or importance_len < S scores every token 1) in position
 * order, then the recent window; else keep = 0..S-1.  keep: int32 [S]
 * (device); count: device int32, the number kept.  One CTA. */
int b2f_evict_keep_indices(const float* importance, int64_t importance_len, int64_t S, int64_t sink,
                           int64_t window, int64_t budget, int32_t* keep, int32_t* count,
                           void* stream);

/* dst[o, i, :] = src[o, keep[i], :] for o < outer, i < n_keep; rows of
 * row_bytes bytes, src [outer, S_src, row], dst [outer, n_keep, row] (the
 * reindexing of [H, S, D] keys/values, streaming_llm.py:129-160 and
 * kv_compression.py:349-355, and of per-token score arrays). */
int b2f_gather_tokens(const void* src, void* dst, int64_t outer, int64_t S_src, int64_t row_bytes,
                      const int32_t* keep, int64_t n_keep, void* stream);

/* Compaction of a paged quantized KV cache (head-major pages [page][Hkv][PS]
 * of D*bits/8 code bytes + D/64 fp32 scales per row) after an eviction
 * decision: for sequence b and i < n_keep[b], token keep[b*keep_ld + i] of
 * the pages named by block_table_src moves to position i of the pages named
 * by block_table_dst (K and V codes and scales, every KV head).  Source and
 * destination pages must be distinct.  The eviction policies of
 * streaming_llm.py:129-160 and kv_compression.py:293-364 applied to the
 * quantized cache instead of full-precision [H, S, D] arrays. */
int b2f_kv_pages_gather(const uint8_t* k_pages, const float* k_scales, const uint8_t* v_pages,
                        const float* v_scales, const int32_t* block_table_src, const int32_t* keep,
                        int64_t keep_ld, const int32_t* n_keep, int64_t max_keep,
                        uint8_t* k_pages_out, float* k_scales_out, uint8_t* v_pages_out,
                        float* v_scales_out, const int32_t* block_table_dst, int64_t max_pages,
                        int64_t B, int64_t Hkv, int64_t D, int64_t page_size, int bits, void* stream);

/* ---- (e) expert parallelism: device halves of dispatch / combine -------- */

/* Replaces the expert-to-rank routing of distributed_experts.py:36-80
 * (ExpertShard.owner_of / DistributedExpertManager) for HBM-resident
 * experts.  `recv` holds W gathered routing segments of seg_bytes each (one
 * per rank, in rank order; the output of an all-gather).  Segment r: T
 * bf16 rows of the normalised hidden state, row pitch row_bytes, at byte 0;
 * int32 top-k expert ids [T, k] at inds_off; float32 scores [T, k] at
 * scores_off.  Assignment a = (r*T + t)*k + j.  This rank owns the global
 * experts [e_begin, e_begin + e_count) of e_total.  Writes a plan over the
 * local experts (same workspace format and size as b2f_moe_plan with
 * A = W*T*k, E = e_count) plus, per assignment: x_row[a] = the assignment's
 * row in `recv` viewed as bf16 [W*seg_bytes/row_bytes, row_bytes/2];
 * wts[a] = its score, or 0 if another rank owns the expert; local[a] = its
 * local expert id, or -1.  Ids outside [0, e_total) set B2F_ERR_INVALID in
 * status_out (device int32, may be NULL). */
int b2f_ep_plan(const void* recv, int64_t seg_bytes, int64_t row_bytes, int64_t inds_off,
                int64_t scores_off, int64_t W, int64_t T, int64_t k, int64_t e_begin,
                int64_t e_count, int64_t e_total, int tile, int32_t* x_row, float* wts,
                int32_t* local, void* workspace, int64_t workspace_bytes,
                int32_t* status_out, void* stream);

/* Per gathered token g < G: out[g, :] = bf16(sum_j wts[g*k+j] * y[g*k+j, :])
 * over the j with local[g*k+j] >= 0 (this rank's share of the weighted
 * expert sum at expert_streaming.py:464-470; 0 where the token has no local
 * expert).  A sum over ranks of `out` (a reduce-scatter) completes the MoE
 * output.  bf16 y [G*k, ldy], out [G, ldo]; H % 8 == 0. */
int b2f_ep_combine_partial(const void* y, int64_t ldy, const float* wts, const int32_t* local,
                           int64_t G, int64_t k, int64_t H, void* out, int64_t ldo, void* stream);

/* ---- (e) expert-parallel decode exchange over NVLink peer memory -------- */
/* The dispatch / combine of distributed_experts.py:36-150's expert partition
 * done by this library's kernels storing into the other GPUs' memory (CUDA
 * IPC mappings of each rank's shared region), in place of the NCCL
 * all-gather / reduce-scatter above.  Region layout (identical on every rank):
 * uint32 flags at flags_off (dispatch [64], combine [64]), W routing segments
 * of seg_bytes at *seg_off (the all-gather's layout, so b2f_ep_plan runs on
 * it unchanged), bf16 combine rows [T][W][H] at *comb_off.  Returns the
 * region's bytes (0 for invalid sizes); the region and the caller's int32
 * control words ctl[4] must be ZERO before the first exchange.  `peers` is a
 * device array of the W regions' base addresses as mapped in this process
 * (entry `rank` = the own region). */
int64_t b2f_ep_p2p_region_bytes(int64_t W, int64_t T, int64_t H, int64_t seg_bytes, int64_t* seg_off,
                                int64_t* comb_off);
/* CUDA IPC of a region for the peer exchange (one process per GPU): export
 * writes the 64-byte handle of the device allocation holding `ptr` and ptr's
 * byte offset in it; import (with the importing rank's device current) maps a
 * peer's allocation into this process for the CURRENT device, enabling peer
 * access, and returns its base (add the exporter's offset); close unmaps. */
int b2f_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);
int b2f_ipc_import(const void* handle, void** base_out);
int b2f_ipc_close(void* base);
/* Dispatch: copies this rank's segment `seg` into slot `rank` of every peer's
 * segment area, writes mask[T][W] (1.0 where rank d owns one of token m's
 * experts under the ExpertShard block partition, else 0) and, once every
 * copy is visible system-wide, raises this rank's dispatch flag in every
 * region with the next exchange number (ctl[0] + 1).  An expert id outside
 * [0, e_total) records B2F_ERR_INVALID in *status_out. */
int b2f_ep_p2p_dispatch(const void* seg, int64_t seg_bytes, const int64_t* peers, int64_t seg_off,
                        int64_t flags_off, int rank, int W, const int32_t* inds, int64_t T, int64_t k,
                        int64_t e_total, float* mask, int32_t* ctl, int32_t* status_out, void* stream);
/* Waits until all W flags of `kind` (0 dispatch, 1 combine) in this rank's
 * region carry the current exchange number ctl[0]; a wait that runs past the
 * wait limit (b2f_set_wait_limit_ns, 2 s by default) records
 * B2F_ERR_TIMEOUT in *status_out and the device status and returns. */
int b2f_ep_p2p_wait(const void* region, int64_t flags_off, int kind, int W, const int32_t* ctl,
                    int32_t* status_out, void* stream);
/* b2f_ep_plan over the segment area of this rank's region (region + seg_off)
 * that first waits, like b2f_ep_p2p_wait, for the W dispatch flags of the
 * current exchange (one launch instead of two; a wait that runs out records
 * B2F_ERR_TIMEOUT in *wait_status). */
int b2f_ep_p2p_plan(const void* region, int64_t seg_off, int64_t flags_off, int64_t seg_bytes, int64_t row_bytes,
                    int64_t inds_off, int64_t scores_off, int W, int64_t T, int64_t k, int64_t e_begin,
                    int64_t e_count, int64_t e_total, int tile, int32_t* x_row, float* wts, int32_t* local,
                    void* workspace, int64_t workspace_bytes, int32_t* status_out, const int32_t* ctl,
                    int32_t* wait_status, void* stream);
/* The owner's completion of the combine once the W combine flags carry the
 * current exchange's number: h = resid + sum_d mask[m,d] * rows[m*W + d]
 * (the combine rows at region + comb_off), resid_out = bf16(h), norm_out =
 * RMSNorm(h) -- b2f_combine_rmsnorm with k = W and the wait folded in. */
int b2f_ep_p2p_combine_rmsnorm(const void* resid, const void* region, int64_t comb_off, int64_t flags_off,
                               const float* mask, int64_t M, int W, const void* weight, float eps, int64_t H,
                               void* resid_out, void* norm_out, const int32_t* ctl, int32_t* wait_status,
                               void* stream);
/* Combine: b2f_ep_combine_partial's weighted sums for the W*T gathered tokens,
 * each stored into the owning rank's combine row (token * W + rank) -- only
 * tokens with a local expert -- then this rank's combine flag is raised in
 * every region.  The owner completes the MoE output with
 * b2f_combine_rmsnorm(resid, rows, mask, T, W, ...). */
int b2f_ep_p2p_combine(const void* y, int64_t ldy, const float* wts, const int32_t* local, int64_t T, int64_t k,
                       int64_t H, const int64_t* peers, int64_t comb_off, int64_t flags_off, int rank, int W,
                       int32_t* ctl, void* stream);

/* ---- (e) expert parallelism over a variable-split all-to-all ---------- */
/* The dispatch / combine halves of distributed_experts.py:36-150's expert
 * partition for prefill-sized batches (one NCCL all_to_all_single of counts,
 * then one of rows, each way).  A dispatched row is [bf16 hidden row H][int32
 * local expert ids k (-1: another rank's)][float32 scores k], padded to
 * b2f_ep_a2a_row_pitch(H, k) bytes (a multiple of 16). */
int64_t b2f_ep_a2a_row_pitch(int64_t H, int64_t k);

/* Pack this rank's T tokens for W ranks: token t goes once to every rank d
 * owning one of its experts (ExpertShard blocks of floor(E/W), the last rank
 * the remainder), at row pos[t*W + d] of `send` (rows grouped by d, token order
 * within d; -1 = not sent); send_counts[d] = rows for d.  x bf16 [T, ldx];
 * inds int32 / scores f32 [T, k] (global ids in [0, e_total), else
 * B2F_ERR_INVALID in status_out).  send holds T*min(W,k) rows. */
int b2f_ep_a2a_dispatch(const void* x, int64_t ldx, const int32_t* inds, const float* scores,
                        int64_t T, int64_t k, int64_t W, int64_t e_total, int64_t H, void* send,
                        int64_t send_bytes, int32_t* pos, int32_t* send_counts,
                        int32_t* status_out, void* stream);

/* MoE plan (as b2f_moe_plan, A = R*k) over R received rows: assignment
 * a = r*k + j of local expert id j of row r, skipped when -1; per assignment
 * x_row[a] = r, wts[a] = its score (0 if skipped), local[a] = the id or -1.
 * The received rows are a bf16 matrix of leading dimension pitch/2 for the
 * expert kernels' x-row index. */
int b2f_ep_a2a_plan(const void* recv, int64_t R, int64_t H, int64_t k, int64_t e_count, int tile,
                    int32_t* x_row, float* wts, int32_t* local, void* workspace,
                    int64_t workspace_bytes, int32_t* status_out, void* stream);

/* out[t] = resid[t] (if non-NULL) + sum over d = 0..W-1 of ret[pos[t*W + d]]
 * (rows the owner ranks returned), f32 accumulation, bf16 out [T, ldo]. */
int b2f_ep_a2a_combine(const void* ret, int64_t ldr, const int32_t* pos, int64_t T, int64_t W,
                       int64_t H, const void* resid, void* out, int64_t ldo, void* stream);

/* ---- smaller ops: Q4_0 GEMV, kernels/ops.py drop-ins, 2-bit requant,
 *      sensitivity fake quantization ------------------------------------- */

/* flash_dequant_gemv_q4 (kernels/flash_dequant.metal:19-49), for nvec input
 * vectors: y[b, m] = sum_n (code(m,n) - 8) * scales[m, n/group_size] * x[b, n].
 * weights uint8 [M, N/2], code 2i in the low nibble of byte i, 2i+1 in the
 * high nibble; scales fp16 [M, N/group_size]; x fp32 [nvec, N]; y fp32
 * [nvec, M]; fp32 accumulation.  group_size a multiple of 32; weights
 * 16-byte aligned. */
int b2f_q4_0_gemv(const uint8_t* weights, const void* scales, const float* x, float* y,
                  int64_t M, int64_t N, int group_size, int64_t nvec, void* stream);

/* kernels/ops.py:48-108 swiglu(gate, up): out = silu(gate) * up computed in
 * fp32, stored in `dtype` (B2F_BF16, B2F_F16 or B2F_F32), n elements. */
int b2f_swiglu(const void* gate, const void* up, void* out, int64_t n, int dtype, void* stream);

/* kernels/ops.py:111-148 moe_dispatch for T tokens: out[t, :] =
 * sum_j expert_outputs_t[selected_ids[t, j], :] * routing_weights[t, j],
 * expert_outputs_t = expert_outputs + t * eo_token_stride elements, each
 * [E, H] of `dtype`; ids int32 [T, k]; weights fp32 [T, k]; out [T, H] of
 * `dtype`; fp32 accumulation.  eo_token_stride 0 shares one [E, H] block. */
int b2f_moe_dispatch(const void* expert_outputs, int64_t eo_token_stride, int64_t E, int64_t H,
                     const int32_t* selected_ids, const float* routing_weights, int64_t T,
                     int64_t k, int dtype, void* out, void* stream);

/* requantize_4bit_to_2bit (mixed_precision.py:130-216), bit-exact: wq uint32
 * [rows, cols_u32] (8 LSB-first nibbles per word), scales/biases [rows,
 * n_groups] of `dtype`; per group of wpg = 8*cols_u32/n_groups codes
 * (a power of two, 4..1024): v = nib*s + b, crumb = clip(rint((v-min)/range*3),
 * 0, 3) with range = max-min (1e-10 if smaller); packed uint8 [rows,
 * 2*cols_u32], crumb j at bits 2*(j%4) of byte j/4; scales2 = fp16(range/3),
 * biases2 = fp16(min), both [rows, n_groups]. */
int b2f_requant_4to2(const uint32_t* wq, int64_t rows, int64_t cols_u32, const void* scales,
                     const void* biases, int dtype, int64_t n_groups, uint8_t* packed,
                     void* scales2, void* biases2, void* stream);

/* dequantize_2bit (mixed_precision.py:219-245): out fp32 [rows,
 * n_values_per_row] = crumb * scale2 + bias2 (fp16 scale/bias [rows, n_groups]). */
int b2f_dequant_2bit(const uint8_t* packed, int64_t packed_ld, const void* scales2,
                     const void* biases2, int64_t n_groups, int64_t rows,
                     int64_t n_values_per_row, float* out, void* stream);

/* _quantize_linears_inplace (layer_quantization.py:461-494) for one tensor of
 * n elements: scale = max(dtype(absmax/qmax), 1e-10), out fp32 =
 * clip(rint(w/scale), qmin, qmax) * scale with (qmin, qmax) = (-8, 7) for
 * bits 4 and (-128, 127) for bits 8.  absmax_out: device fp32, receives
 * max|w|. */
int b2f_fake_quant_sym(const void* w, int dtype, int64_t n, int bits, float* out,
                       float* absmax_out, void* stream);

/* ---- decode-step glue around the hot path (Qwen3-MoE-shaped decoder) ----- */

/* MoE combine + residual + RMSNorm in one pass (expert_streaming.py:464-470
 * `y = (y * scores[..., None]).sum(-2)` and the shared-expert add, then the
 * next RMSNorm):  h = resid + sum_j scores[m,j] * y[m*k+j];  resid_out =
 * bf16(h); norm_out = bf16(weight * h * rsqrt(mean(h^2) + eps)).  y may be
 * NULL (plain RMSNorm); scores may be NULL (every score 1, e.g. k = 1 for an
 * already combined expert-parallel output).  resid_out may alias resid.
 * H % 8 == 0, H <= 8192. */
/* b2f_combine_rmsnorm with the residual update taken from split-K partials:
 * h = resid + sum_r partial[r][m][:] (nsplit fp32 planes [M, H], 16-byte
 * aligned); resid_out = bf16(h); norm_out = RMSNorm(h). */
int b2f_combine_rmsnorm_partials(const void* resid, const float* partial, int nsplit, int64_t M,
                                 const void* weight, float eps, int64_t H, void* resid_out,
                                 void* norm_out, void* stream);

/* b2f_qk_norm_rope_kv_append reading the q/k/v projection as split-K partials
 * (nsplit fp32 planes [B, (Hq+2Hkv)*D]): the row is bf16(sum of the planes),
 * the value the projection's bf16 output would hold. */
int b2f_qk_norm_rope_kv_append_partials(const float* qkv_partial, int nsplit, int64_t B, int64_t Hq,
                                        int64_t Hkv, int64_t D, const void* q_norm,
                                        const void* k_norm, float eps, float rope_theta,
                                        const int32_t* positions, void* q_out, uint8_t* k_codes,
                                        float* k_scales, uint8_t* v_codes, float* v_scales,
                                        const int32_t* block_table, int64_t max_pages,
                                        int64_t page_size, int bits, void* stream);

int b2f_combine_rmsnorm(const void* resid, const void* y, const float* scores, int64_t M,
                        int64_t k, const void* weight, float eps, int64_t H, void* resid_out,
                        void* norm_out, void* stream);

/* Per token: q heads RMSNorm(q_norm)+RoPE -> q_out [B,Hq,D]; k heads
 * RMSNorm(k_norm)+RoPE then the reference KV quantizer (bf16 arithmetic,
 * group 64) into head-major page slot positions[b]; v heads quantized as is.
 * qkv: bf16 [B, (Hq+2*Hkv)*D].  D = 128; bits in {2,4,8}.  This is the append
 * path of QuantizedKVEntry.append (quantized_kv_cache.py:284-309) fused with
 * the attention prologue. */
int b2f_qk_norm_rope_kv_append(const void* qkv, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                               const void* q_norm, const void* k_norm, float eps,
                               float rope_theta, const int32_t* positions, void* q_out,
                               uint8_t* k_codes, float* k_scales, uint8_t* v_codes,
                               float* v_scales, const int32_t* block_table, int64_t max_pages,
                               int64_t page_size, int bits, void* stream);

/* Router of the MoE block (expert_streaming.py:439-472): gates =
 * softmax(x.wr^T + bias), top-k (ties to the lower id), scores = gates of the
 * top-k, renormalised to sum 1 if renorm.  x bf16 [T,H] (H % 8 == 0); wr bf16
 * [E,H] (E <= 256); bias f32 [E] or NULL; logits_ws f32 [T,E] caller workspace (holds the
 * gates afterwards); inds int32 [T,k]; scores f32 [T,k]. */
int b2f_moe_route_topk(const void* x, int64_t T, int64_t H, const void* wr, const float* bias,
                       int64_t E, int64_t k, int renorm, float* logits_ws, int32_t* inds,
                       float* scores, void* stream);

/* Gate kinds of the _ex routers. */
#define B2F_GATE_SOFTMAX 0 /* gates = softmax over the experts (expert_streaming.py:440) */
#define B2F_GATE_SIGMOID 1 /* gates = sigmoid per expert (DeepSeek-V3-style routing) */

/* b2f_moe_route_topk with the gate kind and the LExI skip of the reference's
 * skip-fallback forward (enable_skip_fallback, expert_streaming.py:439-462):
 * with skip_threshold > 0, slot 0 (the largest gate) is kept and slot j >= 1
 * gets score 0 when top1 > skip_threshold * score_j; renorm then divides the
 * scores by their sum when that sum is positive (:459-460).  The reference
 * takes top1 from an argpartition whose order inside the top-k MLX does not
 * define; here slots are in descending gate order, so slot 0 is the largest. */
int b2f_moe_route_topk_ex(const void* x, int64_t T, int64_t H, const void* wr, const float* bias,
                          int64_t E, int64_t k, int renorm, int gating, float skip_threshold,
                          float* logits_ws, int32_t* inds, float* scores, void* stream);

/* b2f_moe_route_plan with the gate kind and skip of b2f_moe_route_topk_ex. */
int b2f_moe_route_plan_ex(const void* x, int64_t T, int64_t H, const void* wr, const float* bias,
                          int64_t E, int64_t k, int renorm, int gating, float skip_threshold,
                          float* logits_ws, int32_t* inds, float* scores, int tile,
                          void* plan_workspace, int64_t plan_workspace_bytes, int32_t* status_out,
                          void* stream);

/* out[t, e] = x[t].wr[e] + bias[e] in f32, then sigmoid if apply_sigmoid: the
 * shared expert's gate sigmoid(shared_expert_gate(x)) of expert_streaming.py:466-470
 * (E = 1), or raw router logits.  x bf16 [T,H] (H % 8 == 0, H <= 8192), wr bf16
 * [E,H] (E <= 256), bias f32 [E] or NULL. */
int b2f_router_logits(const void* x, int64_t T, int64_t H, const void* wr, const float* bias,
                      int64_t E, int apply_sigmoid, float* out, void* stream);

/* Greedy next token: out[m] = argmax_v x[m, v] (ties to the lower index). */
int b2f_argmax_rows(const void* x, int64_t M, int64_t V, int32_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B2F_H_ */
