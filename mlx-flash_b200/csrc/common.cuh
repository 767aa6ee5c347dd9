// Shared helpers for the sm_100a kernels of libb200flash.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2f.h"

namespace b2f {

// Records the CUDA error text for b2f_last_error_string() (thread local).
void set_last_cuda_error(cudaError_t e);

inline int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return B2F_ERR_CUDA;
  }
  return B2F_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- programmatic dependent launch --------------------------------------
// With the calling thread's launch policy on (b2f_set_launch_pdl), kernels
// are launched with programmatic stream serialization: a kernel may be
// scheduled while the one before it in the stream finishes its last wave.
// Every kernel so launched calls pdl_enter() before it touches global
// memory: griddepcontrol.wait returns once the previous kernel has completed
// and its writes are visible, then griddepcontrol.launch_dependents lets
// the next kernel be scheduled.  Waiting before triggering keeps the chain
// transitive -- when kernel n may start, kernel n-2 has completed -- so a
// kernel may read data written two or more launches back before its wait.
// Both instructions do nothing in a normal launch.
int& launch_pdl_policy();

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
  pdl_wait();
  pdl_trigger();
}

// kern<<<grid, block, smem, st>>>(args...) under the launch policy; B2F_OK or
// B2F_ERR_CUDA (with the CUDA error text recorded)
template <typename... P, typename... A>
inline int launch_kernel(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (launch_pdl_policy()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<A&&>(args)...);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return B2F_ERR_CUDA;
  }
  return check_launch();
}

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// ---- element types -----------------------------------------------------
// Each tag converts its storage type to float and rounds a float back with
// IEEE round-to-nearest-even (the rounding MLX applies after an f32 op).
struct TagBF16 {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f(T v) { return __bfloat162float(v); }
  static __device__ __forceinline__ T from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) { return to_f(from_f(v)); }
};
struct TagF16 {
  using T = __half;
  static __device__ __forceinline__ float to_f(T v) { return __half2float(v); }
  static __device__ __forceinline__ T from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round(float v) { return to_f(from_f(v)); }
};
struct TagF32 {
  using T = float;
  static __device__ __forceinline__ float to_f(T v) { return v; }
  static __device__ __forceinline__ T from_f(float v) { return v; }
  static __device__ __forceinline__ float round(float v) { return v; }
};

// ---- warp reductions ---------------------------------------------------
template <int WIDTH>
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int WIDTH>
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int WIDTH>
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---- bit helpers -------------------------------------------------------
// lop3: (a & b) | c
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// ---- legacy warp-level tensor-core MMA (register operands) -------------
// D[16x8] += A[16x16] * B[16x8], fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4],
                                              const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace b2f

namespace b2f {
// ---- TMA bulk copies and mbarriers (sm_90+ PTX, used on sm_100a) ---------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory (no multicast); completion
// is signalled as transaction bytes on `bar`.  16-byte aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// ---- bounded waits: limit, sticky timeout status, test control ----------
// One copy per translation unit (the library is built without relocatable
// device code); the host reaches every unit's copy through b2f_device_status,
// b2f_set_wait_limit_ns and b2f_set_producer_stall.
//   b2f_tu_status   B2F_ERR_TIMEOUT once any kernel of the unit had a bounded
//                   wait give up (sticky until read with clear)
//   b2f_tu_wait_ns  the default wait limit (2 s)
//   b2f_tu_stall    test control, 0 in normal operation: non-zero makes the
//                   producer warps issue no copies, so the consumers' waits
//                   run out (how the tests exercise the timeout paths)
static __device__ int32_t b2f_tu_status = 0;
static __device__ unsigned long long b2f_tu_wait_ns = 2000000000ull;
static __device__ int32_t b2f_tu_stall = 0;

__device__ __forceinline__ bool producers_stalled() { return *const_cast<volatile int32_t*>(&b2f_tu_stall) != 0; }

// A kernel whose bounded wait gave up: the call's own status word (if any)
// and the unit's sticky status both get B2F_ERR_TIMEOUT.
__device__ __forceinline__ void report_timeout(int32_t* err) {
  if (err) atomicExch(err, B2F_ERR_TIMEOUT);
  atomicExch(&b2f_tu_status, B2F_ERR_TIMEOUT);
}

// Waits for the phase with the given parity; gives up after `limit_ns`
// (0: the unit's limit, 2 s by default) and returns false instead of
// spinning forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  if (limit_ns == 0) limit_ns = *const_cast<volatile unsigned long long*>(&b2f_tu_wait_ns);
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > limit_ns) return false;
  }
  return true;
}
// mbar_wait_bounded for a thread that has nothing else to do while it waits
// (a producer whose ring is full): backs off between polls so the spinning
// thread leaves the issue slots to the warps doing the work.
__device__ __forceinline__ bool mbar_wait_bounded_backoff(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  if (limit_ns == 0) limit_ns = *const_cast<volatile unsigned long long*>(&b2f_tu_wait_ns);
  const uint64_t t0 = global_ns();
  uint32_t ns = 32;
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > limit_ns) return false;
    __nanosleep(ns);
    if (ns < 256) ns <<= 1;
  }
  return true;
}
// Host accessor of this unit's controls (one per .cu file with bounded
// waits): op 0 reads the status into *v, 1 reads and clears it, 2 sets the
// wait limit to *v ns, 3 sets the producer stall to *v.
#define B2F_DEFINE_WAIT_CONTROLS(NAME)                                                            \
  int b2f_wait_controls_##NAME(int op, long long* v) {                                           \
    cudaError_t e = cudaSuccess;                                                                  \
    if (op == 0 || op == 1) {                                                                     \
      int32_t st = 0;                                                                             \
      e = cudaMemcpyFromSymbol(&st, b2f_tu_status, sizeof(st));                                   \
      *v = st;                                                                                    \
      if (e == cudaSuccess && op == 1) {                                                          \
        const int32_t z = 0;                                                                      \
        e = cudaMemcpyToSymbol(b2f_tu_status, &z, sizeof(z));                                     \
      }                                                                                           \
    } else if (op == 2) {                                                                         \
      const unsigned long long ns = (unsigned long long)(*v);                                     \
      e = cudaMemcpyToSymbol(b2f_tu_wait_ns, &ns, sizeof(ns));                                    \
    } else if (op == 3) {                                                                         \
      const int32_t on = int32_t(*v);                                                             \
      e = cudaMemcpyToSymbol(b2f_tu_stall, &on, sizeof(on));                                      \
    }                                                                                             \
    return e == cudaSuccess ? 0 : -1;                                                             \
  }

// named barrier over the first `nthreads` threads of the CTA (id 1)
__device__ __forceinline__ void named_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}
}  // namespace b2f
