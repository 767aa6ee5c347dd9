// (e) Expert-parallel decode exchange over NVLink peer memory.
//
// The same two exchanges as the all-gather / reduce-scatter form in ep.cu
// (the reference's distributed-expert plan, distributed_experts.py:36-150,
// with every expert resident in some GPU's HBM), done by this library's own
// kernels writing straight into the other GPUs' memory instead of by NCCL:
//
//   dispatch  b2f_ep_p2p_dispatch: every rank copies its routing segment
//             {x rows, top-k ids, scores} into slot `rank` of every peer's
//             segment area, then raises its dispatch flag in every peer;
//             the same launch writes this rank's combine mask (which ranks
//             own one of each token's experts);
//   wait      b2f_ep_p2p_wait: the rank waits (bounded) until all W flags of
//             the exchange carry this exchange's number;
//   partial   b2f_ep_p2p_combine: per gathered token the score-weighted sum
//             of its local expert outputs, stored directly into the owning
//             rank's combine area at row (token * W + this rank) -- only for
//             tokens with at least one local expert -- then the combine flag
//             is raised in every peer;
//   combine   the owner sums its W rows per token, weighted by the mask
//             (b2f_combine_rmsnorm with k = W: residual add and RMSNorm in the
//             same pass).
//
// Shared region of every rank (the same byte layout on every rank; peers'
// regions are mapped into this process by CUDA IPC and passed as a table of
// W base addresses):
//   [flags_off]  uint32 dispatch flags [64] then combine flags [64]: flag s =
//                the number of the last exchange rank s completed towards this
//                rank;
//   [seg_off]    W routing segments of seg_bytes (the all-gather's layout);
//   [comb_off]   bf16 combine rows [T][W][H].
// Control words local to each rank (int32 [4], zero at start): [0] the number
// of the current exchange, [1] / [2] arrival counters of the dispatch /
// combine CTAs (each launch leaves them zero).
//
// Ordering: each writing thread fences at system scope after its stores; the
// last CTA to arrive raises the flags with release stores; waiters poll with
// acquire loads.  A rank overwrites a peer's segment slot (combine row) for
// the next exchange only after it waited for that peer's combine (dispatch)
// flag of the current one, which the peer raises after it finished reading
// the slot (row), so one region serves every layer.  Every wait gives up
// after the unit's wait limit and reports B2F_ERR_TIMEOUT instead of
// spinning forever.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
#include "norm.cuh"
#include "plan.cuh"

namespace b2f {

constexpr int P2P_MAX_W = 64;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t* p2p_flag(int64_t base, int64_t flags_off, int kind, int src) {
  return reinterpret_cast<uint32_t*>(base + flags_off) + kind * P2P_MAX_W + src;
}
__device__ __forceinline__ int p2p_owner(int e, int per, int W) { return min(e / per, W - 1); }

// The last CTA of a launch to arrive raises flag `kind` of this rank in every
// peer with the exchange number; the arrival counter is left zero.
__device__ __forceinline__ void p2p_arrive_and_signal(const int64_t* peers, int64_t flags_off, int kind, int rank,
                                                      int W, int32_t* ctl, bool new_exchange) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned total = gridDim.x * gridDim.y;
    const unsigned old = atomicAdd(reinterpret_cast<unsigned*>(ctl + 1 + kind), 1u);
    if (old == total - 1) {
      __threadfence_system();
      ctl[1 + kind] = 0;
      uint32_t seq = uint32_t(*const_cast<volatile int32_t*>(ctl));
      if (new_exchange) {
        seq += 1u;
        *const_cast<volatile int32_t*>(ctl) = int32_t(seq);
      }
      for (int d = 0; d < W; ++d) st_release_sys(p2p_flag(peers[d], flags_off, kind, rank), seq);
    }
  }
}

struct P2PDispatch {
  const uint4* seg;       // this rank's routing segment (seg_bytes / 16 words)
  const int64_t* peers;   // [W] region base addresses as mapped in this process
  int64_t seg_off, seg_bytes, flags_off;
  int rank, W;
  int32_t* ctl;
  // combine mask of this rank's tokens: mask[m*W + d] = 1 if rank d owns one
  // of token m's experts, else 0
  const int32_t* inds;
  int T, k, e_total;
  float* mask;
  int32_t* status;
};

// grid (blocks per peer, W): block (x, d) copies its share of the segment to
// peer d; the blocks of y == rank write the mask instead.
__global__ void __launch_bounds__(256) ep_p2p_dispatch_kernel(const P2PDispatch p) {
  const int d = blockIdx.y;
  if (d != p.rank) {
    uint4* dst = reinterpret_cast<uint4*>(p.peers[d] + p.seg_off + int64_t(p.rank) * p.seg_bytes);
    const int64_t n = p.seg_bytes / 16;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
      dst[i] = p.seg[i];
    __threadfence_system();
  } else {
    const int per = p.e_total / p.W;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.T * p.W; i += gridDim.x * blockDim.x) {
      const int m = i / p.W, dd = i - m * p.W;
      float f = 0.f;
      for (int j = 0; j < p.k; ++j) {
        const int e = p.inds[int64_t(m) * p.k + j];
        if (e < 0 || e >= p.e_total) {
          if (p.status) atomicExch(p.status, B2F_ERR_INVALID);
          continue;
        }
        if (p2p_owner(e, per, p.W) == dd) f = 1.f;
      }
      p.mask[i] = f;
    }
  }
  p2p_arrive_and_signal(p.peers, p.flags_off, 0, p.rank, p.W, p.ctl, true);
}

// Threads s < W of the block wait (bounded) for flag s to reach the current
// exchange number ctl[0]; then the whole block passes a barrier.  Called at
// the start of the kernels that read what the exchange delivered.
__device__ __forceinline__ void p2p_block_wait(const uint32_t* flags, int W, const int32_t* ctl, int32_t* status) {
  const int s = threadIdx.x;
  if (s < W) {
    const uint32_t seq = uint32_t(*const_cast<const volatile int32_t*>(ctl));
    if (int32_t(ld_acquire_sys(flags + s) - seq) < 0) {
      const uint64_t limit = *const_cast<volatile unsigned long long*>(&b2f_tu_wait_ns);
      const uint64_t t0 = global_ns();
      uint32_t ns = 32;
      while (int32_t(ld_acquire_sys(flags + s) - seq) < 0) {
        if (global_ns() - t0 > limit) {
          report_timeout(status);
          break;
        }
        __nanosleep(ns);
        if (ns < 512) ns <<= 1;
      }
    }
  }
  __syncthreads();
}

// The MoE plan over the W routing segments once the dispatch flags of every
// rank carry this exchange's number (b2f_ep_plan with the wait folded in).
__global__ void __launch_bounds__(1024) ep_p2p_plan_kernel(const GatheredExperts src, int A, int E, int tile,
                                                           char* ws, PlanLayout L, int32_t* status_out,
                                                           const uint32_t* flags, int W, const int32_t* ctl,
                                                           int32_t* wait_status) {
  pdl_wait();
  p2p_block_wait(flags, W, ctl, wait_status);
  pdl_trigger();
  moe_plan_block(src, A, E, tile, ws, L, status_out);
}

// The owner's completion of the combine once every rank's combine flag
// carries this exchange's number: h = resid + sum_d mask[m,d] * rows[m*W+d],
// then RMSNorm (b2f_combine_rmsnorm with k = W and the wait folded in).
__global__ void __launch_bounds__(256) ep_p2p_combine_rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ resid, const __nv_bfloat16* __restrict__ rows, const float* __restrict__ mask,
    int W, const __nv_bfloat16* __restrict__ w, float eps, int H, __nv_bfloat16* __restrict__ resid_out,
    __nv_bfloat16* __restrict__ norm_out, const uint32_t* flags, const int32_t* ctl, int32_t* wait_status) {
  pdl_wait();
  p2p_block_wait(flags, W, ctl, wait_status);
  pdl_trigger();
  combine_rmsnorm_block(resid, rows, mask, W, w, eps, H, resid_out, norm_out, nullptr, 0, 0);
}

// One CTA of up to 64 threads: thread s waits for flag s of `kind` to reach
// the current exchange number.
__global__ void __launch_bounds__(64) ep_p2p_wait_kernel(const uint32_t* flags, int W, const int32_t* ctl,
                                                         int32_t* status) {
  const int s = threadIdx.x;
  if (s < W) {
    const uint32_t seq = uint32_t(*const_cast<const volatile int32_t*>(ctl));
    if (int32_t(ld_acquire_sys(flags + s) - seq) < 0) {
      const uint64_t limit = *const_cast<volatile unsigned long long*>(&b2f_tu_wait_ns);
      const uint64_t t0 = global_ns();
      uint32_t ns = 32;
      while (int32_t(ld_acquire_sys(flags + s) - seq) < 0) {
        if (global_ns() - t0 > limit) {
          report_timeout(status);
          break;
        }
        __nanosleep(ns);
        if (ns < 512) ns <<= 1;
      }
    }
  }
  __syncthreads();
}

struct P2PCombine {
  const __nv_bfloat16* y;  // expert outputs, one row per gathered assignment
  int64_t ldy;
  const float* wts;
  const int32_t* local;  // local expert of each gathered assignment, -1 if another rank's
  int k, H, T;
  const int64_t* peers;
  int64_t comb_off, flags_off;
  int rank, W;
  int32_t* ctl;
};

// One CTA per gathered token g = src * T + m: the weighted sum of its local
// expert outputs, stored into rank src's combine row (m * W + rank).
__global__ void __launch_bounds__(256) ep_p2p_combine_kernel(const P2PCombine p) {
  const int64_t g = blockIdx.x;
  const int src = int(g / p.T), m = int(g - int64_t(src) * p.T);
  __shared__ float w_s[32];
  __shared__ int j_s[32];
  __shared__ int n_s;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int j = 0; j < p.k; ++j) {
      const int64_t a = g * p.k + j;
      if (p.local[a] >= 0) {
        w_s[n] = p.wts[a];
        j_s[n] = j;
        ++n;
      }
    }
    n_s = n;
  }
  __syncthreads();
  const int n = n_s;
  if (n > 0) {
    uint4* dst = reinterpret_cast<uint4*>(p.peers[src] + p.comb_off +
                                          (int64_t(m) * p.W + p.rank) * int64_t(p.H) * 2);
    for (int v = threadIdx.x; v < p.H / 8; v += blockDim.x) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int i = 0; i < n; ++i) {
        const float sc = w_s[i];
        const uint4 yy = reinterpret_cast<const uint4*>(p.y + (g * p.k + j_s[i]) * p.ldy)[v];
        const __nv_bfloat162* y2 = reinterpret_cast<const __nv_bfloat162*>(&yy);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[2 * q] += sc * __low2float(y2[q]);
          acc[2 * q + 1] += sc * __high2float(y2[q]);
        }
      }
      uint4 o;
      uint32_t* o32 = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) o32[q] = pack_bf16x2(acc[2 * q], acc[2 * q + 1]);
      dst[v] = o;
    }
    __threadfence_system();
  }
  p2p_arrive_and_signal(p.peers, p.flags_off, 1, p.rank, p.W, p.ctl, false);
}

B2F_DEFINE_WAIT_CONTROLS(p2p)

}  // namespace b2f

using namespace b2f;

namespace b2f {
// cuMemGetAddressRange through the runtime's driver entry point: the base of
// the device allocation that holds a pointer (the unit of CUDA IPC)
static std::mutex g_range_mu;
static PFN_cuMemGetAddressRange_v3020 g_range = nullptr;
static int get_range_fn() {
  std::lock_guard<std::mutex> lock(g_range_mu);
  if (g_range) return B2F_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  const cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
    set_last_cuda_error(e == cudaSuccess ? cudaErrorNotSupported : e);
    return B2F_ERR_CUDA;
  }
  g_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  return B2F_OK;
}
}  // namespace b2f

extern "C" {

int b2f_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return B2F_ERR_INVALID;
  int rc = get_range_fn();
  if (rc != B2F_OK) return rc;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return B2F_ERR_INVALID;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return B2F_ERR_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = int64_t(reinterpret_cast<uintptr_t>(ptr) - uintptr_t(base));
  return B2F_OK;
}

int b2f_ipc_import(const void* handle, void** base_out) {
  if (!handle || !base_out) return B2F_ERR_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return B2F_ERR_CUDA;
  }
  return B2F_OK;
}

int b2f_ipc_close(void* base) {
  if (!base) return B2F_ERR_INVALID;
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return B2F_ERR_CUDA;
  }
  return B2F_OK;
}

int64_t b2f_ep_p2p_region_bytes(int64_t W, int64_t T, int64_t H, int64_t seg_bytes, int64_t* seg_off,
                                int64_t* comb_off) {
  if (W <= 0 || W > P2P_MAX_W || T <= 0 || H <= 0 || H % 8 != 0 || seg_bytes <= 0 || seg_bytes % 16 != 0) return 0;
  const int64_t so = 1024;  // flags: 2 x 64 uint32, padded
  const int64_t co = align_up(so + W * seg_bytes, 256);
  if (seg_off) *seg_off = so;
  if (comb_off) *comb_off = co;
  return align_up(co + T * W * H * 2, 256);
}

int b2f_ep_p2p_dispatch(const void* seg, int64_t seg_bytes, const int64_t* peers, int64_t seg_off,
                        int64_t flags_off, int rank, int W, const int32_t* inds, int64_t T, int64_t k,
                        int64_t e_total, float* mask, int32_t* ctl, int32_t* status_out, void* stream) {
  if (W <= 0 || W > P2P_MAX_W || rank < 0 || rank >= W || T < 0 || k <= 0 || k > 32 || e_total < W)
    return B2F_ERR_INVALID;
  if (seg_bytes <= 0 || seg_bytes % 16 != 0 || seg_off < 0 || flags_off < 0 || flags_off % 4 != 0)
    return B2F_ERR_INVALID;
  if (!seg || !peers || !ctl || !mask || (T > 0 && !inds)) return B2F_ERR_INVALID;
  if (!aligned(seg, 16) || seg_off % 16 != 0) return B2F_ERR_ALIGN;
  if (T * W > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  P2PDispatch p;
  p.seg = static_cast<const uint4*>(seg);
  p.peers = peers;
  p.seg_off = seg_off;
  p.seg_bytes = seg_bytes;
  p.flags_off = flags_off;
  p.rank = rank;
  p.W = W;
  p.ctl = ctl;
  p.inds = inds;
  p.T = int(T);
  p.k = int(k);
  p.e_total = int(e_total);
  p.mask = mask;
  p.status = status_out;
  // enough blocks per peer that the copy is spread over many SMs (a segment
  // of a 64-token decode batch at H 2048 is ~260 KB)
  const int64_t words = seg_bytes / 16;
  int per_peer = int(std::min<int64_t>(16, (words + 255) / 256));
  if (per_peer < 1) per_peer = 1;
  ep_p2p_dispatch_kernel<<<dim3(unsigned(per_peer), unsigned(W)), 256, 0, as_stream(stream)>>>(p);
  return check_launch();
}

int b2f_ep_p2p_wait(const void* region, int64_t flags_off, int kind, int W, const int32_t* ctl, int32_t* status_out,
                    void* stream) {
  if (W <= 0 || W > P2P_MAX_W || !(kind == 0 || kind == 1) || flags_off < 0 || flags_off % 4 != 0)
    return B2F_ERR_INVALID;
  if (!region || !ctl) return B2F_ERR_INVALID;
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(static_cast<const char*>(region) + flags_off) +
                          kind * P2P_MAX_W;
  ep_p2p_wait_kernel<<<1, 64, 0, as_stream(stream)>>>(flags, W, ctl, status_out);
  return check_launch();
}

int b2f_ep_p2p_plan(const void* region, int64_t seg_off, int64_t flags_off, int64_t seg_bytes, int64_t row_bytes,
                    int64_t inds_off, int64_t scores_off, int W, int64_t T, int64_t k, int64_t e_begin,
                    int64_t e_count, int64_t e_total, int tile, int32_t* x_row, float* wts, int32_t* local,
                    void* workspace, int64_t workspace_bytes, int32_t* status_out, const int32_t* ctl,
                    int32_t* wait_status, void* stream) {
  if (W <= 0 || W > P2P_MAX_W || T < 0 || k <= 0 || k > 32 || e_count <= 0 || e_begin < 0 ||
      e_begin + e_count > e_total)
    return B2F_ERR_INVALID;
  if (tile < 8 || tile > 256 || tile % 8 != 0) return B2F_ERR_INVALID;
  if (row_bytes <= 0 || seg_bytes <= 0 || seg_bytes % row_bytes != 0) return B2F_ERR_INVALID;
  if (inds_off < 0 || scores_off < 0 || inds_off % 4 || scores_off % 4 || flags_off < 0 || flags_off % 4)
    return B2F_ERR_ALIGN;
  if (inds_off + 4 * T * k > seg_bytes || scores_off + 4 * T * k > seg_bytes || T * row_bytes > inds_off)
    return B2F_ERR_INVALID;
  const int64_t A = int64_t(W) * T * k;
  if (A > 0x3fffffff || e_count > 65535 || W * (seg_bytes / row_bytes) > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  PlanLayout L = plan_layout(A, e_count, tile);
  if (!workspace || workspace_bytes < L.total) return B2F_ERR_WORKSPACE;
  if (!region || !ctl || (A > 0 && (!x_row || !wts || !local))) return B2F_ERR_INVALID;
  const char* recv = static_cast<const char*>(region) + seg_off;
  if (!aligned(workspace, 16) || !aligned(recv, 16)) return B2F_ERR_ALIGN;
  GatheredExperts src;
  src.recv = recv;
  src.seg_bytes = seg_bytes;
  src.inds_off = inds_off;
  src.scores_off = scores_off;
  src.seg_rows = seg_bytes / row_bytes;
  src.T = int(T);
  src.k = int(k);
  src.e_begin = int(e_begin);
  src.e_total = int(e_total);
  src.x_row = x_row;
  src.wts = wts;
  src.local = local;
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(static_cast<const char*>(region) + flags_off);
  return launch_kernel(ep_p2p_plan_kernel, dim3{1}, dim3{1024}, 0, as_stream(stream), src, int(A), int(e_count),
                       tile, static_cast<char*>(workspace), L, status_out, flags, W, ctl, wait_status);
}

int b2f_ep_p2p_combine_rmsnorm(const void* resid, const void* region, int64_t comb_off, int64_t flags_off,
                               const float* mask, int64_t M, int W, const void* weight, float eps, int64_t H,
                               void* resid_out, void* norm_out, const int32_t* ctl, int32_t* wait_status,
                               void* stream) {
  if (M < 0 || H <= 0 || W <= 0 || W > P2P_MAX_W) return B2F_ERR_INVALID;
  if (H % 8 != 0 || H > CMB_CHUNKS * 8 * 256) return B2F_ERR_UNSUPPORTED;
  if (M == 0) return B2F_OK;
  if (!resid || !region || !mask || !weight || !norm_out || !ctl) return B2F_ERR_INVALID;
  const char* rows = static_cast<const char*>(region) + comb_off;
  if (comb_off % 16 != 0 || flags_off < 0 || flags_off % 4 != 0 || !aligned(resid, 16) || !aligned(rows, 16) ||
      !aligned(weight, 16) || !aligned(norm_out, 16) || (resid_out && !aligned(resid_out, 16)))
    return B2F_ERR_ALIGN;
  const int threads = int(H / 8) < 256 ? int(((H / 8) + 31) / 32 * 32) : 256;
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(static_cast<const char*>(region) + flags_off) +
                          P2P_MAX_W;  // the combine flags
  return launch_kernel(ep_p2p_combine_rmsnorm_kernel, dim3{unsigned(M)}, dim3{unsigned(threads < 64 ? 64 : threads)},
                       0, as_stream(stream), static_cast<const __nv_bfloat16*>(resid),
                       reinterpret_cast<const __nv_bfloat16*>(rows), mask, W,
                       static_cast<const __nv_bfloat16*>(weight), eps, int(H),
                       static_cast<__nv_bfloat16*>(resid_out), static_cast<__nv_bfloat16*>(norm_out), flags, ctl,
                       wait_status);
}

int b2f_ep_p2p_combine(const void* y, int64_t ldy, const float* wts, const int32_t* local, int64_t T, int64_t k,
                       int64_t H, const int64_t* peers, int64_t comb_off, int64_t flags_off, int rank, int W,
                       int32_t* ctl, void* stream) {
  if (W <= 0 || W > P2P_MAX_W || rank < 0 || rank >= W || T < 0 || k <= 0 || k > 32 || H <= 0 || H % 8 != 0 ||
      ldy < H)
    return B2F_ERR_INVALID;
  if (comb_off < 0 || comb_off % 16 != 0 || flags_off < 0 || flags_off % 4 != 0) return B2F_ERR_ALIGN;
  if (ldy % 8) return B2F_ERR_ALIGN;
  if (!peers || !ctl || (T > 0 && (!y || !wts || !local))) return B2F_ERR_INVALID;
  if (T > 0 && !aligned(y, 16)) return B2F_ERR_ALIGN;
  if (W * T > 0x7fffffff) return B2F_ERR_UNSUPPORTED;
  P2PCombine p;
  p.y = static_cast<const __nv_bfloat16*>(y);
  p.ldy = ldy;
  p.wts = wts;
  p.local = local;
  p.k = int(k);
  p.H = int(H);
  p.T = int(T);
  p.peers = peers;
  p.comb_off = comb_off;
  p.flags_off = flags_off;
  p.rank = rank;
  p.W = W;
  p.ctl = ctl;
  const int threads = int(H / 8 < 256 ? ((H / 8 + 31) / 32) * 32 : 256);
  // a launch with no tokens still raises the flags (one CTA)
  const unsigned blocks = T > 0 ? unsigned(W * T) : 1u;
  if (T == 0) p.T = 1, p.k = 0;
  ep_p2p_combine_kernel<<<blocks, threads, 0, as_stream(stream)>>>(p);
  return check_launch();
}

}  // extern "C"
