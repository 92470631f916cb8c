// Shared device helpers for the Qwen3 decode kernels (sm_100a).
//
// Weight layout ("packed"): a [n, k] BF16 matrix (PyTorch [out, in], y = x W^T) is cut into
// 16 KiB blocks of 128 rows x 64 columns. Block (g, kb) holds rows 128g..128g+127 and columns
// 64kb..64kb+63; blocks are stored group-major (g outer, kb inner), so a row group's blocks are
// contiguous and one bulk copy moves one block. Inside a block each row is 128 bytes (eight 16-byte
// chunks) and chunk c of row r is stored at position c ^ (r & 7): the 128-byte swizzle that the
// tensor cores' K-major shared-memory operand format uses, and a bank-conflict-free pattern for
// the CUDA-core GEMV, whose eight lanes of a row read the eight chunks of that row.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qd {

constexpr int kBlockRows = 128;
constexpr int kBlockCols = 64;
constexpr int kBlockBytes = kBlockRows * kBlockCols * 2;  // 16384
constexpr uint64_t kWaitLimitNs = 1000000000ull;          // 1 s bound on every device-side wait

// error bits written to the caller's err word (see include/qd_decode.h)
constexpr int kErrWaitFull = 1;
constexpr int kErrWaitEmpty = 2;
constexpr int kErrDrain = 4;
constexpr int kErrDep = 32;  // a wait for another CTA's results (persistent step kernel) timed out
constexpr int kErrSmem = 64;  // dynamic shared memory not aligned as the kernel's layout requires

__host__ __device__ __forceinline__ int64_t packed_offset_elems(int64_t n, int64_t k, int64_t kblocks) {
  const int64_t g = n >> 7, r = n & 127, kb = k >> 6, c = (k & 63) >> 3, e = k & 7;
  return ((g * kblocks + kb) * kBlockRows + r) * kBlockCols + ((c ^ (r & 7)) << 3) + e;
}

// Stream-K partition of T blocks over G CTAs: CTA c owns blocks [begin(c), begin(c+1)).
__host__ __device__ __forceinline__ int64_t part_begin(int64_t T, int G, int c) {
  return (int64_t)c * T / G;
}
// The CTA that owns block b (largest c with begin(c) <= b).
__host__ __device__ __forceinline__ int part_owner(int64_t T, int G, int64_t b) {
  return (int)(((b + 1) * (int64_t)G - 1) / T);
}

__device__ __forceinline__ float bf16_to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier + bulk copy (TMA)
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: true when the phase with `parity` completed; false (and err |= code) after
// kWaitLimitNs without it. Never spins forever.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0 && globaltimer() - t0 > kWaitLimitNs) {
      if (err) atomicOr(err, code);
      return false;
    }
  }
}

// mbar_wait that also gives up at once when another CTA has raised `abort` (polled every 64 tries), and
// raises it itself when its own limit expires, so one expired wait ends the whole grid quickly.
__device__ __forceinline__ bool mbar_wait_abort(uint32_t bar, uint32_t parity, int* err, int code, int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*reinterpret_cast<volatile int*>(abort)) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        if (err) atomicOr(err, code);
        atomicExch(abort, 1);
        return false;
      }
    }
  }
}

// Orders this thread's generic-proxy global accesses with async-proxy (TMA / bulk copy) accesses: a
// writer issues it before publishing data a bulk copy will read, the reader after acquiring the flag.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// One-dimensional bulk copy global -> this CTA's shared memory, completing on `bar`. No multicast.
// `policy` is an L2 cache policy (createpolicy) for the source lines.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}
// Fire-and-forget prefetch of a global range into L2 (no completion tracking).
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------- programmatic dependent launch
// wait: block until the preceding kernel in the stream has completed and its writes are visible
// (a no-op when the launch carried no programmatic dependency).
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// L2-only loads (bypass L1, which is not coherent across SMs) of data produced by other CTAs or
// by the previous kernel. Compiler intrinsics rather than volatile asm, so independent loads are
// issued back to back; they are never moved across a barrier or fence (those clobber memory).
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint2 ld_cg_v2(const void* p) { return __ldcg(reinterpret_cast<const uint2*>(p)); }
__device__ __forceinline__ float ld_cg_f32(const float* p) { return __ldcg(p); }
__device__ __forceinline__ int64_t ld_cg_s64(const int64_t* p) {
  return (int64_t)__ldcg(reinterpret_cast<const long long*>(p));
}

// gpu-scope release add / acquire load for the inter-CTA completion counters and tickets. The
// pattern is: every thread writes, CTA barrier, one thread releases (release is cumulative over what
// the barrier made visible to it); the reader acquires in one thread, then a CTA barrier.
__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_volatile(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait (one thread) until *cnt >= target: one acquire load per try (the load orders the caller's
// later reads after the releases it observed), the abort flag and the clock read only every 64 tries.
// Returns false when another CTA raised *abort, or when kWaitLimitNs passed (then err |= code and
// *abort = 1).
__device__ __forceinline__ bool wait_count_ge(const int* cnt, int target, int* abort, int* err, int code) {
  if (ld_acquire(cnt) >= target) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire(cnt) >= target) return true;
    if ((i & 63u) == 0) {
      if (abort && ld_volatile(abort)) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        if (err) atomicOr(err, code);
        if (abort) atomicExch(abort, 1);
        return false;
      }
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace qd
