// Tensor-core (tcgen05) skinny GEMM for 16..64 activation rows, sm_100a.
//
// Swap-AB: y^T[128 weight rows x N] += W[128 x 16] . x^T[16 x N] per tcgen05.mma (M = 128, N = the
// batch padded to a multiple of 16, K = 16), BF16 operands from shared memory, fp32 accumulators in
// tensor memory (TMEM). Both operands use the 128-byte-swizzled K-major layout that the packed weight
// blocks already have, so one bulk copy of a 16 KiB block is a ready A operand; the activations are
// packed once per projection into the same layout (qd_pack_act: RMSNorm applied, rows zero-padded),
// [k/64][N][64], so one bulk copy of N x 128 bytes is the matching B operand.
//
// Warp roles in a CTA of 320 threads: warp 8 produces (weight block + activation tile per ring stage,
// mbarrier complete_tx), warp 9 issues the MMAs (one thread) into two alternating TMEM accumulators
// and commits each stage back to its ring slot, warps 0-7 are the epilogue: per row-group segment they
// read the accumulator (tcgen05.ld 32x32b, warp w reads TMEM lanes 32(w % 4).. and half of the
// columns), then run the same split-K flush and fused epilogues as the CUDA-core kernel
// (qd_gemv_dev.cuh). The work partition (stream-K over blocks) is the CUDA-core kernel's.
// Development timeline (built only with -DQD_TC_TRACE): %globaltimer stamps per CTA into a buffer set
// with qd_tc_trace_set; slot layout in tc_gemv_kernel.
#ifdef QD_TC_TRACE
namespace qd {
static __device__ unsigned long long* g_tc_trace;
}
#define QD_FLUSH_HOOK(k, flags, tid)                                                                   \
  do {                                                                                               \
    if (g_tc_trace && (tid) == 0) g_tc_trace[blockIdx.x * 64 + (flags)[3] + (k)] = globaltimer();     \
  } while (0)
#define TC_STAMP(k)                                                            \
  do {                                                                         \
    if (g_tc_trace) g_tc_trace[blockIdx.x * 64 + (k)] = globaltimer();         \
  } while (0)
#else
#define TC_STAMP(k) \
  do {              \
  } while (0)
#endif
#include "qd_gemv_dev.cuh"
#include "qd_plan.h"
#include "qd_umma.cuh"

namespace qd {

constexpr int kTcThreads = kThreads + 32;  // 8 epilogue warps + producer (8) + MMA issuer (9)

struct TcLayout {
  int ring, stage, red, wsum, lmv, lmi, flags, aux, bars, tslot, total;
};

__host__ __device__ inline int tal(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline TcLayout tc_layout(int N, int nst) {
  TcLayout L;
  L.stage = kBlockBytes + N * 128;  // weight block + activation tile (both 1024-B aligned)
  L.ring = 0;
  int off = nst * L.stage;
  L.red = off;
  off += N * kBlockRows * 4;
  L.wsum = off;
  off += N * kConsumerWarps * 4 + 64;
  L.lmv = off;
  off += tal(N * 4, 16);
  L.lmi = off;
  off += tal(N * 4, 16);
  L.flags = off;
  off += 16;
  L.aux = off;
  off += 512 * 4;
  L.bars = tal(off, 8);
  off = L.bars + (2 * nst + 4) * 8;
  L.tslot = off;
  off += 16;
  L.total = tal(off, 1024);
  return L;
}

template <int N>
constexpr int tmem_cols() {  // two accumulators of N fp32 columns, power of two >= 32
  return 2 * N <= 32 ? 32 : (2 * N <= 64 ? 64 : (2 * N <= 128 ? 128 : 256));
}

template <int N, int MODE, bool DEFER = false>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(1024) char smem_raw[];
  // the 128-byte swizzle is a function of the shared address: operand tiles must sit on 1 KiB boundaries
  char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const TcLayout Ly = tc_layout(N, a.nst);
  const int nst = a.nst;
  char* ring = smem + Ly.ring;
  float* red = reinterpret_cast<float*>(smem + Ly.red);
  float* wsum = reinterpret_cast<float*>(smem + Ly.wsum);
  float* lmv = reinterpret_cast<float*>(smem + Ly.lmv);
  int* lmi = reinterpret_cast<int*>(smem + Ly.lmi);
  int* flags = reinterpret_cast<int*>(smem + Ly.flags);
  float* aux = reinterpret_cast<float*>(smem + Ly.aux);
  const uint32_t bars = smem_u32(smem + Ly.bars);
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (nst + s); };
  auto accf_bar = [&](int i) { return bars + 8u * (2 * nst + i); };
  auto acce_bar = [&](int i) { return bars + 8u * (2 * nst + 2 + i); };
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + Ly.tslot);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  const int64_t b_begin = part_begin(a.total, a.grid, cta), b_end = part_begin(a.total, a.grid, cta + 1);
  const int64_t xtile = (int64_t)N * 128;  // bytes of one activation tile

  if (tid == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(accf_bar(i), 1);
      mbar_init(acce_bar(i), kConsumerWarps);
    }
    fence_mbar_init();
    flags[0] = 0;
    flags[1] = 0;
  }
  if (tid < N) {
    lmv[tid] = -INFINITY;
    lmi[tid] = 0x7fffffff;
  }
  if (warp == kConsumerWarps + 1) {  // the MMA warp owns the tensor memory
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(tmem_cols<N>()));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) TC_STAMP(0);

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const int nblk = (int)(b_end - b_begin);
      const char* wsrc = a.w + b_begin * (int64_t)kBlockBytes;
      const int first = nblk < nst ? nblk : nst;
      const int ahead = a.prefetch;
      int pf = 0;
      // weights never depend on the preceding kernel: L2 prefetch and the first ring's worth of copies
      // go out before waiting on it
      for (; pf < nblk && pf < first + ahead; ++pf) prefetch_l2(wsrc + pf * (int64_t)kBlockBytes, kBlockBytes);
      for (int i = 0; i < first; ++i) {
        mbar_arrive_expect_tx(full_bar(i), (uint32_t)(kBlockBytes + xtile));
        bulk_g2s(smem_u32(ring + i * Ly.stage), wsrc + i * (int64_t)kBlockBytes, kBlockBytes, full_bar(i), pol);
      }
      TC_STAMP(1);
      grid_dep_wait();
      TC_STAMP(2);
      int kb = (int)(b_begin % a.kblocks);
      for (int i = 0; i < first; ++i) {
        bulk_g2s(smem_u32(ring + i * Ly.stage + kBlockBytes), a.x_packed + kb * xtile, (uint32_t)xtile, full_bar(i),
                 pol);
        if (++kb == a.kblocks) kb = 0;
      }
      int issued = first, slot = 0, round = 1;
      for (int i = first; i < nblk; ++i) {
        for (; pf < nblk && pf <= i + ahead; ++pf) prefetch_l2(wsrc + pf * (int64_t)kBlockBytes, kBlockBytes);
        if (!mbar_wait(empty_bar(slot), (round - 1) & 1, a.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(full_bar(slot), (uint32_t)(kBlockBytes + xtile));
        bulk_g2s(smem_u32(ring + slot * Ly.stage), wsrc + i * (int64_t)kBlockBytes, kBlockBytes, full_bar(slot), pol);
        bulk_g2s(smem_u32(ring + slot * Ly.stage + kBlockBytes), a.x_packed + kb * xtile, (uint32_t)xtile,
                 full_bar(slot), pol);
        if (++kb == a.kblocks) kb = 0;
        ++issued;
        if (++slot == nst) {
          slot = 0;
          ++round;
        }
      }
      flags[0] = issued;
      TC_STAMP(3);
    }
  } else if (warp == kConsumerWarps + 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(N);
      const int nblk = (int)(b_end - b_begin);
      bool ok = true;
      int buf = 0, uses[2] = {0, 0}, slot = 0, fph = 0;
      int kb = (int)(b_begin % a.kblocks);
      for (int i = 0; i < nblk; ++i) {
        const bool seg_start = (i == 0) || (kb == 0);
        const bool seg_end = (kb == a.kblocks - 1) || (i == nblk - 1);
        if (seg_start && uses[buf] > 0 && ok) ok = mbar_wait(acce_bar(buf), (uses[buf] - 1) & 1, a.err, kErrWaitFull);
        if (ok) ok = mbar_wait(full_bar(slot), fph, a.err, kErrWaitFull);
        tc_fence_after();
        if (ok) {
          const uint32_t sa = smem_u32(ring + slot * Ly.stage), sb = sa + kBlockBytes;
#pragma unroll
          for (int j = 0; j < 4; ++j)  // K = 64 per block, 16 per MMA: +32 bytes along the swizzled row
            umma_bf16(tmem + buf * N, umma_desc_sw128(sa + 32 * j), umma_desc_sw128(sb + 32 * j), idesc,
                      (seg_start && j == 0) ? 0u : 1u);
        }
        umma_commit(empty_bar(slot));  // frees the slot once these MMAs have read it
        if (seg_end) {
          umma_commit(accf_bar(buf));
          ++uses[buf];
          buf ^= 1;
        }
        if (++slot == nst) {
          slot = 0;
          fph ^= 1;
        }
        if (++kb == a.kblocks) kb = 0;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (256 threads)
    grid_dep_wait();
    grid_dep_launch();
    if constexpr (MODE == MODE_QKV) qkv_prologue(a, aux, flags, tid);
    if (tid == 0) TC_STAMP(6);
    int n_seg = 0;
    bool ok = true;
    int buf = 0, fph[2] = {0, 0};
    const int q = warp & 3, half = warp >> 2;
    int64_t seg_first = b_begin;
    int g = (int)(b_begin / a.kblocks);
    int kb = (int)(b_begin % a.kblocks) - 1;
    for (int64_t b = b_begin; b < b_end; ++b) {
      if (++kb == a.kblocks) {
        kb = 0;
        ++g;
      }
      const bool seg_end = (kb == a.kblocks - 1) || (b == b_end - 1);
      if (!seg_end) continue;
      if (ok) ok = mbar_wait(accf_bar(buf), fph[buf], a.err, kErrWaitFull);
      fph[buf] ^= 1;
      tc_fence_after();
      if (tid == 0 && n_seg < 7) TC_STAMP(8 + 8 * n_seg);
      // row r = 32q + lane of the group; this warp's half of the N batch columns
#pragma unroll
      for (int c8 = 0; c8 < N / 16; ++c8) {
        float v[8];
        const int col = half * (N / 2) + 8 * c8;
        tmem_ld8(tmem + ((uint32_t)(32 * q) << 16) + buf * N + col, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 8; ++e) red[(col + e) * kBlockRows + 32 * q + lane] = v[e];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar(buf));
      buf ^= 1;
      if (tid == 0) {
        if (n_seg < 7) TC_STAMP(9 + 8 * n_seg);
        flags[3] = 8 + 8 * (n_seg < 7 ? n_seg : 6);  // trace slot base of this segment's flush phases
      }
      named_bar(kBarConsumers, kConsumers);
      flush_segment<N, MODE, DEFER>(a, g, seg_first, b, cta, red, wsum, lmv, lmi, aux, flags, tid);
      if (tid == 0 && n_seg < 7) TC_STAMP(13 + 8 * n_seg);
      ++n_seg;
      seg_first = b + 1;
    }
    if constexpr (MODE == MODE_LM) lm_global_argmax<N>(a, cta, wsum, lmv, lmi, flags, tid);
    (void)ok;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kConsumerWarps + 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols<N>()));
  if (tid == 0) {  // no bulk copy may still be writing shared memory
    const int issued = flags[0];
    for (int it = issued > nst ? issued - nst : 0; it < issued; ++it)
      if (!mbar_wait(full_bar(it % nst), (it / nst) & 1, a.err, kErrDrain)) break;
  }
}

// ------------------------------------------------------------------ activation packing
struct PackActArgs {
  const __nv_bfloat16* x;
  int64_t ldx, k;
  const __nv_bfloat16* norm_w;
  float eps;
  __nv_bfloat16* xpk;
  int n_pad;
};

// One CTA per real activation row: optional Qwen3RMSNorm, then the row's 64-column chunks go to
// xpk[(kb * n_pad + m) * 64 + ((c ^ (m & 7)) * 8) + e] - the swizzled K-major tile layout.
__global__ void __launch_bounds__(256) pack_act_kernel(const __grid_constant__ PackActArgs a) {
  __shared__ float wsum[8];
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k8 = (int)(a.k >> 3);
  float rstd = 1.f;
  if (a.norm_w) {
    float sq = 0.f;
    for (int q = tid; q < k8; q += 256) {
      const uint4 v = ld_cg_v4(a.x + m * a.ldx + q * 8);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = bf_lo(u[e]), hi = bf_hi(u[e]);
        sq = fmaf(lo, lo, sq);
        sq = fmaf(hi, hi, sq);
      }
    }
    sq = warp_sum(sq);
    if (lane == 0) wsum[warp] = sq;
    __syncthreads();
    float ss = 0.f;
#pragma unroll
    for (int w8 = 0; w8 < 8; ++w8) ss += wsum[w8];
    rstd = 1.0f / sqrtf(ss / (float)a.k + a.eps);
  }
  for (int q = tid; q < k8; q += 256) {
    uint4 v = ld_cg_v4(a.x + m * a.ldx + q * 8);
    if (a.norm_w) {
      const uint4 wv = *reinterpret_cast<const uint4*>(a.norm_w + q * 8);
      const uint32_t xu[4] = {v.x, v.y, v.z, v.w};
      const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = bf16r(bf_lo(wu[e]) * bf16r(bf_lo(xu[e]) * rstd));
        const float hi = bf16r(bf_hi(wu[e]) * bf16r(bf_hi(xu[e]) * rstd));
        o[e] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
      }
      v = make_uint4(o[0], o[1], o[2], o[3]);
    }
    const int kb = q >> 3, c = q & 7;
    *reinterpret_cast<uint4*>(a.xpk + ((int64_t)kb * a.n_pad + m) * 64 + ((c ^ (m & 7)) << 3)) = v;
  }
}

// The residual add a QD_EPI_RES_SUMS projection left behind, then the packing of qd_pack_act: row m of x
// becomes bf16(x + bf16(sum)) (written back to x), its sums are cleared for the next projection, and the
// row is RMSNorm-ed (optional) into the packed operand. One CTA of 256 threads per row.
struct PackResArgs {
  __nv_bfloat16* x;
  int64_t ldx, k;
  int64_t* fxs;  // [m_act][k]
  const __nv_bfloat16* norm_w;
  float eps;
  __nv_bfloat16* xpk;
  int n_pad;
};

__global__ void __launch_bounds__(256) pack_act_res_kernel(const __grid_constant__ PackResArgs a) {
  __shared__ float wsum[8];
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k8 = (int)(a.k >> 3);
  // this thread's first chunks q = tid + 256 j (j < kCh): residual, sums and norm weights all requested
  // before any is used, the new values kept in registers for the normalising pass; a row wider than
  // kCh chunks per thread (k > 4096) takes the rest chunk by chunk and re-reads its values
  constexpr int kCh = 2;
  uint4 xv[kCh], wv[kCh];
  longlong2 sv[kCh][4];
  float sq = 0.f;
  {
#pragma unroll
    for (int j = 0; j < kCh; ++j) {
      const int q = j * 256 + tid;
      if (q < k8) {
        xv[j] = ld_cg_v4(a.x + m * a.ldx + q * 8);
        const longlong2* sp = reinterpret_cast<const longlong2*>(a.fxs + m * a.k + q * 8);
#pragma unroll
        for (int e = 0; e < 4; ++e) sv[j][e] = __ldcg(sp + e);
        if (a.norm_w) wv[j] = *reinterpret_cast<const uint4*>(a.norm_w + q * 8);
      }
    }
#pragma unroll
    for (int j = 0; j < kCh; ++j) {
      const int q = j * 256 + tid;
      if (q >= k8) continue;
      const uint32_t ru[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = bf16r(bf_lo(ru[e]) + bf16r(fx_to_float(sv[j][e].x)));
        const float hi = bf16r(bf_hi(ru[e]) + bf16r(fx_to_float(sv[j][e].y)));
        o[e] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
        sq = fmaf(lo, lo, sq);
        sq = fmaf(hi, hi, sq);
      }
      xv[j] = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(a.x + m * a.ldx + q * 8) = xv[j];
      longlong2* sp = reinterpret_cast<longlong2*>(a.fxs + m * a.k + q * 8);
#pragma unroll
      for (int e = 0; e < 4; ++e) sp[e] = make_longlong2(0, 0);
    }
  }
  if (k8 > kCh * 256) {  // the remaining chunks of a wide row
    for (int q = kCh * 256 + tid; q < k8; q += 256) {
      const uint4 v = ld_cg_v4(a.x + m * a.ldx + q * 8);
      longlong2* sp = reinterpret_cast<longlong2*>(a.fxs + m * a.k + q * 8);
      const longlong2 s4[4] = {__ldcg(sp), __ldcg(sp + 1), __ldcg(sp + 2), __ldcg(sp + 3)};
      const uint32_t ru[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = bf16r(bf_lo(ru[e]) + bf16r(fx_to_float(s4[e].x)));
        const float hi = bf16r(bf_hi(ru[e]) + bf16r(fx_to_float(s4[e].y)));
        o[e] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
        sq = fmaf(lo, lo, sq);
        sq = fmaf(hi, hi, sq);
      }
      *reinterpret_cast<uint4*>(a.x + m * a.ldx + q * 8) = make_uint4(o[0], o[1], o[2], o[3]);
#pragma unroll
      for (int e = 0; e < 4; ++e) sp[e] = make_longlong2(0, 0);
    }
  }
  float rstd = 1.f;
  if (a.norm_w) {
    sq = warp_sum(sq);
    if (lane == 0) wsum[warp] = sq;
    __syncthreads();
    float ss = 0.f;
#pragma unroll
    for (int w8 = 0; w8 < 8; ++w8) ss += wsum[w8];
    rstd = 1.0f / sqrtf(ss / (float)a.k + a.eps);
  }
  for (int q = tid; q < k8; q += 256) {
    const int j = (q - tid) >> 8;  // which register chunk, when the row fits in registers
    uint4 v, w;
    if (k8 <= kCh * 256) {
      v = j == 0 ? xv[0] : xv[1];
      w = j == 0 ? wv[0] : wv[1];
    } else {
      v = ld_cg_v4(a.x + m * a.ldx + q * 8);  // this thread's own write above
      if (a.norm_w) w = *reinterpret_cast<const uint4*>(a.norm_w + q * 8);
    }
    if (a.norm_w) {
      const uint32_t xu[4] = {v.x, v.y, v.z, v.w};
      const uint32_t wu[4] = {w.x, w.y, w.z, w.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = bf16r(bf_lo(wu[e]) * bf16r(bf_lo(xu[e]) * rstd));
        const float hi = bf16r(bf_hi(wu[e]) * bf16r(bf_hi(xu[e]) * rstd));
        o[e] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
      }
      v = make_uint4(o[0], o[1], o[2], o[3]);
    }
    const int kb = q >> 3, c = q & 7;
    *reinterpret_cast<uint4*>(a.xpk + ((int64_t)kb * a.n_pad + m) * 64 + ((c ^ (m & 7)) << 3)) = v;
  }
}

// The QKV epilogue (the decode QKV GEMV's arithmetic: BF16 projection output, per-head RMSNorm with
// the sum of squares taken per 32 rows and the 4 slices added in order, q_norm / k_norm, RoPE at the
// decode position with every product rounded to BF16, q store, K/V append) applied to the fixed-point
// sums a QD_EPI_STORE_SUMS projection left, which it clears. One CTA of 128 threads (one per dimension)
// per (head, row).
struct QkvSumsArgs {
  int64_t* sums;  // [m_act][(nq + 2 nkv) * 128]
  int64_t lds;
  const __nv_bfloat16 *qn, *kn, *cos, *sin;
  const int64_t* pos;
  int64_t cap;
  int nq, nkv;
  float eps;
  __nv_bfloat16 *q_out, *k_cache, *v_cache;
  int64_t cs_b, cs_h;
  int* err;
};

__global__ void __launch_bounds__(128) qkv_rope_sums_kernel(const __grid_constant__ QkvSumsArgs a) {
  __shared__ float wsq[4];
  __shared__ float ys[128];
  grid_dep_wait();
  grid_dep_launch();
  const int g = blockIdx.x, m = blockIdx.y, r = threadIdx.x, lane = r & 31, w = r >> 5;
  // everything that does not depend on the position in one round trip: the position, this element's
  // sum, its norm weight; then the RoPE row
  int64_t* sp = a.sums + (int64_t)m * a.lds + (int64_t)g * 128 + r;
  const int64_t p = ld_cg_s64(a.pos);
  const long long sraw = __ldcg(sp);
  const bool vhead = g >= a.nq + a.nkv;
  const __nv_bfloat16 nwb = vhead ? __float2bfloat16_rn(0.f) : (g < a.nq ? a.qn[r] : a.kn[r]);
  const bool in = p >= 0 && p < a.cap;  // the same for every thread
  float c = 0.f, sn = 0.f;
  if (in && !vhead) {
    c = bf16_to_f(a.cos[p * 128 + r]);
    sn = bf16_to_f(a.sin[p * 128 + r]);
  }
  const float v = bf16r(fx_to_float(sraw));
  *sp = 0;  // the sums start the next projection clear
  if (!in) {  // flagged, nothing written
    if (r == 0 && g == 0 && m == 0 && a.err) atomicOr(a.err, QD_DEVERR_POS);
    return;
  }
  if (vhead) {  // V head: into the cache as is
    a.v_cache[(int64_t)m * a.cs_b + (int64_t)(g - a.nq - a.nkv) * a.cs_h + p * 128 + r] = __float2bfloat16_rn(v);
    return;
  }
  const float sq = warp_sum(v * v);
  if (lane == 0) wsq[w] = sq;
  __syncthreads();
  const float var = (wsq[0] + wsq[1] + wsq[2] + wsq[3]) / 128.0f;
  const float rstd = 1.0f / sqrtf(var + a.eps);
  const float y = bf16r(bf16_to_f(nwb) * bf16r(v * rstd));
  ys[r] = y;
  __syncthreads();
  const float yp = ys[r ^ 64];
  // q*cos + rotate_half(q)*sin with every product a BF16 tensor (rotate_half = cat(-q2, q1))
  const float rot = (r < 64) ? bf16r(-yp * sn) : bf16r(yp * sn);
  const __nv_bfloat16 o = __float2bfloat16_rn(bf16r(y * c) + rot);
  if (g < a.nq)
    a.q_out[((int64_t)m * a.nq + g) * 128 + r] = o;
  else
    a.k_cache[(int64_t)m * a.cs_b + (int64_t)(g - a.nq) * a.cs_h + p * 128 + r] = o;
}

// ------------------------------------------------------------------ host side
static int tc_ctas_per_sm() {
  const int c = env_int("QD_TC_CTAS_PER_SM", 1);
  return c < 1 ? 1 : (c > 4 ? 4 : c);
}

// L2 prefetch lookahead of the weight stream, in 16 KiB blocks. Off by default: on B200 the ring of
// bulk copies alone keeps this kernel at the same rate (measured 0 / 8 / 16 / 32 blocks).
static int tc_prefetch_blocks() {
  const int v = env_int("QD_TC_PREFETCH", 0);
  return v < 0 ? 0 : (v > 64 ? 64 : v);
}

static int tc_nst(int N) {
  const int cps = tc_ctas_per_sm();
  const int budget = cps == 1 ? 227 * 1024 : 228 * 1024 / cps - 1024;  // 1 KiB reserved per CTA
  // 4 stages: the same rate as 12 (the ring is not the limit) in about half the shared memory, so
  // the next kernel's CTA can be resident beside this one and start its prologue under PDL
  int nst = env_int("QD_TC_STAGES", 4);
  if (nst > 12) nst = 12;
  while (nst > 1 && tc_layout(N, nst).total + 1024 > budget) --nst;  // + base alignment slack
  return nst;
}

static bool tc_plan(int64_t n_rows, int64_t k, int n_pad, int grid_hint, Plan* p) {
  if (n_pad != 16 && n_pad != 32 && n_pad != 48 && n_pad != 64) return false;
  // one CTA per SM (the ring takes most of shared memory); the partition does not depend on the batch
  if (!make_plan(n_rows, k, 8, grid_hint > 0 ? grid_hint : host_sm_count() * tc_ctas_per_sm(), p)) return false;
  const int smax = p->smax, g = p->grid;
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  p->off_tickets = take(p->groups * 4);
  p->off_lm_ticket = take(4);
  p->off_cta_val = take((int64_t)n_pad * g * 4);
  p->off_cta_idx = take((int64_t)n_pad * g * 4);
  p->off_partials = take(p->groups * smax * n_pad * kBlockRows * 4);
  p->bytes = off;
  p->nst = tc_nst(n_pad);
  return p->nst >= 2;
}

template <int N, int MODE, bool DEFER = false>
static int tc_launch_nm(const GemvArgs& a, int pdl, cudaStream_t stream) {
  auto kern = tc_gemv_kernel<N, MODE, DEFER>;
  const int smem = tc_layout(N, a.nst).total + 1024;  // + alignment slack
  if (int rc = set_max_dynamic_smem((const void*)kern, smem)) return rc;
  return launch_kernel((const void*)kern, dim3(a.grid), dim3(kTcThreads), smem, pdl, stream, (void*)&a);
}

template <int MODE, bool DEFER = false>
static int tc_launch_mode(const GemvArgs& a, int N, int pdl, cudaStream_t stream) {
  switch (N) {
    case 16: return tc_launch_nm<16, MODE, DEFER>(a, pdl, stream);
    case 32: return tc_launch_nm<32, MODE, DEFER>(a, pdl, stream);
    case 48: return tc_launch_nm<48, MODE, DEFER>(a, pdl, stream);
    case 64: return tc_launch_nm<64, MODE, DEFER>(a, pdl, stream);
  }
  return set_error(QD_ERR_UNSUPPORTED, "n_pad %d not in {16, 32, 48, 64}", N);
}

static int tc_launch(const GemvArgs& a, int mode, int N, int pdl, cudaStream_t stream) {
  switch (mode) {
    case MODE_STORE: return tc_launch_mode<MODE_STORE>(a, N, pdl, stream);
    case MODE_RES: return tc_launch_mode<MODE_RES>(a, N, pdl, stream);
    case MODE_SWIGLU: return tc_launch_mode<MODE_SWIGLU>(a, N, pdl, stream);
    case MODE_QKV: return tc_launch_mode<MODE_QKV>(a, N, pdl, stream);
    case MODE_LM: return tc_launch_mode<MODE_LM>(a, N, pdl, stream);
  }
  return set_error(QD_ERR_ARG, "unknown epilogue %d", mode);
}

static int tc_common(GemvArgs& a, const void* xpk, int n_pad, int m_act, const void* w, int64_t n_rows, int64_t k,
                     int grid, void* scratch, int64_t scratch_bytes, int* err) {
  Plan p;
  if (!tc_plan(n_rows, k, n_pad, grid, &p))
    return set_error(QD_ERR_UNSUPPORTED, "tc plan: n=%lld k=%lld n_pad=%d (n%%128, k%%64, n_pad in 16..64 step 16)",
                     (long long)n_rows, (long long)k, n_pad);
  if (p.grid != grid) return set_error(QD_ERR_ARG, "grid %d does not match the plan (%d)", grid, p.grid);
  if (!scratch || scratch_bytes < p.bytes)
    return set_error(QD_ERR_SCRATCH, "scratch %lld B < %lld B", (long long)scratch_bytes, (long long)p.bytes);
  if (!xpk || !w || !aligned16(xpk) || !aligned16(w)) return set_error(QD_ERR_ARG, "xpk / weights: null or unaligned");
  if (m_act < 1 || m_act > n_pad) return set_error(QD_ERR_ARG, "m_act must be in 1..n_pad");
  a = GemvArgs{};
  a.x_packed = static_cast<const char*>(xpk);
  a.w = static_cast<const char*>(w);
  a.n = n_rows;
  a.n_valid = n_rows;
  a.k = k;
  a.kblocks = (int)(k / kBlockCols);
  a.total = p.total;
  a.grid = p.grid;
  a.nst = p.nst;
  a.m_act = m_act;
  a.prefetch = tc_prefetch_blocks();
  char* sc = static_cast<char*>(scratch);
  a.tickets = reinterpret_cast<int*>(sc + p.off_tickets);
  a.lm_ticket = reinterpret_cast<int*>(sc + p.off_lm_ticket);
  a.cta_val = reinterpret_cast<float*>(sc + p.off_cta_val);
  a.cta_idx = reinterpret_cast<int*>(sc + p.off_cta_idx);
  a.partials = reinterpret_cast<float*>(sc + p.off_partials);
  a.smax = p.smax;
  a.err = err;
  return QD_OK;
}

}  // namespace qd

using namespace qd;

extern "C" int qd_pack_act(const void* x, int64_t ldx, int m_act, int n_pad, int64_t k, const void* norm_w, float eps,
                           void* xpk, int pdl, cudaStream_t stream) {
  if (!x || !xpk || !aligned16(x) || !aligned16(xpk) || (norm_w && !aligned16(norm_w)))
    return set_error(QD_ERR_ARG, "pack_act: null or unaligned pointer");
  if (m_act < 1 || m_act > n_pad || k % kBlockCols || ldx < k || ldx % 8)
    return set_error(QD_ERR_ARG, "pack_act: bad sizes");
  PackActArgs a = {};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.k = k;
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  a.xpk = static_cast<__nv_bfloat16*>(xpk);
  a.n_pad = n_pad;
  return launch_kernel((const void*)pack_act_kernel, dim3(m_act), dim3(256), 0, pdl, stream, &a);
}

extern "C" int qd_pack_act_res(void* x, int64_t ldx, int m_act, int n_pad, int64_t k, void* fx_sums,
                               const void* norm_w, float eps, void* xpk, int pdl, cudaStream_t stream) {
  if (!x || !xpk || !fx_sums || !aligned16(x) || !aligned16(xpk) || !aligned16(fx_sums) ||
      (norm_w && !aligned16(norm_w)))
    return set_error(QD_ERR_ARG, "pack_act_res: null or unaligned pointer");
  if (m_act < 1 || m_act > n_pad || k % kBlockCols || ldx < k || ldx % 8)
    return set_error(QD_ERR_ARG, "pack_act_res: bad sizes");
  PackResArgs a = {};
  a.x = static_cast<__nv_bfloat16*>(x);
  a.ldx = ldx;
  a.k = k;
  a.fxs = static_cast<int64_t*>(fx_sums);
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  a.xpk = static_cast<__nv_bfloat16*>(xpk);
  a.n_pad = n_pad;
  return launch_kernel((const void*)pack_act_res_kernel, dim3(m_act), dim3(256), 0, pdl, stream, &a);
}

extern "C" int qd_qkv_rope_sums(void* sums, int64_t lds, int m_act, int nq_heads, int nkv_heads, const void* q_norm,
                                const void* k_norm, float eps, const void* cos, const void* sin, const int64_t* pos,
                                int64_t cap, void* q_out, void* k_cache, void* v_cache, int64_t cs_b, int64_t cs_h,
                                int* err, int pdl, cudaStream_t stream) {
  if (!sums || !q_norm || !k_norm || !cos || !sin || !pos || !q_out || !k_cache || !v_cache)
    return set_error(QD_ERR_ARG, "qkv_rope_sums: null pointer");
  if (m_act < 1 || m_act > 65535 || nq_heads < 1 || nkv_heads < 1 || lds < (int64_t)(nq_heads + 2 * nkv_heads) * 128 ||
      cap < 1 || cs_h < cap * 128 || cs_b < (int64_t)nkv_heads * cs_h)
    return set_error(QD_ERR_ARG, "qkv_rope_sums: bad sizes");
  QkvSumsArgs a = {};
  a.sums = static_cast<int64_t*>(sums);
  a.lds = lds;
  a.qn = static_cast<const __nv_bfloat16*>(q_norm);
  a.kn = static_cast<const __nv_bfloat16*>(k_norm);
  a.cos = static_cast<const __nv_bfloat16*>(cos);
  a.sin = static_cast<const __nv_bfloat16*>(sin);
  a.pos = pos;
  a.cap = cap;
  a.nq = nq_heads;
  a.nkv = nkv_heads;
  a.eps = eps;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.cs_b = cs_b;
  a.cs_h = cs_h;
  a.err = err;
  return launch_kernel((const void*)qkv_rope_sums_kernel, dim3(nq_heads + 2 * nkv_heads, m_act), dim3(128), 0, pdl,
                       stream, &a);
}

extern "C" int qd_tc_gemv_plan(int64_t n, int64_t k, int n_pad, int grid_hint, int* grid, int64_t* scratch_bytes) {
  Plan p;
  if (!tc_plan(n, k, n_pad, grid_hint, &p))
    return set_error(QD_ERR_UNSUPPORTED, "tc plan: n=%lld k=%lld n_pad=%d", (long long)n, (long long)k, n_pad);
  if (grid) *grid = p.grid;
  if (scratch_bytes) *scratch_bytes = p.bytes;
  return QD_OK;
}

extern "C" int qd_tc_gemv(const void* xpk, int n_pad, int m_act, const void* w_packed, int64_t n, int64_t k, void* out,
                          int64_t ldo, const void* res, int64_t ldr, int epilogue, int grid, void* scratch,
                          int64_t scratch_bytes, int* err, int pdl, cudaStream_t stream) {
  GemvArgs a;
  if (int rc = tc_common(a, xpk, n_pad, m_act, w_packed, n, k, grid, scratch, scratch_bytes, err)) return rc;
  if (!out) return set_error(QD_ERR_ARG, "null out");
  int mode;
  if (epilogue == QD_EPI_STORE) {
    mode = MODE_STORE;
    if (ldo < n) return set_error(QD_ERR_ARG, "ldo < n");
  } else if (epilogue == QD_EPI_RES) {
    mode = MODE_RES;
    if (!res || ldo < n || ldr < n) return set_error(QD_ERR_ARG, "residual epilogue needs res, ldo/ldr >= n");
  } else if (epilogue == QD_EPI_SWIGLU) {
    mode = MODE_SWIGLU;
    if (ldo < n / 2) return set_error(QD_ERR_ARG, "ldo < n/2");
  } else if (epilogue == QD_EPI_SWIGLU_PACKED) {
    mode = MODE_SWIGLU;
    if (!aligned16(out)) return set_error(QD_ERR_ARG, "packed out must be 16-byte aligned");
    a.out_npad = n_pad;
  } else if (epilogue == QD_EPI_STORE_SUMS) {
    // the projection output stays as fixed-point sums for a following kernel (qd_qkv_rope_sums)
    if (!aligned16(out)) return set_error(QD_ERR_ARG, "sums must be 16-byte aligned");
    a.fx = static_cast<int64_t*>(out);
    return tc_launch_mode<MODE_STORE, true>(a, n_pad, pdl, stream);
  } else if (epilogue == QD_EPI_RES_SUMS) {
    // the residual add is left to the next qd_pack_act_res: out = fixed-point sums [m_act][n] int64
    if (!aligned16(out)) return set_error(QD_ERR_ARG, "sums must be 16-byte aligned");
    a.fx = static_cast<int64_t*>(out);
    return tc_launch_mode<MODE_RES, true>(a, n_pad, pdl, stream);
  } else {
    return set_error(QD_ERR_ARG, "unknown epilogue %d", epilogue);
  }
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.res = static_cast<const __nv_bfloat16*>(res);
  a.ldr = ldr;
  return tc_launch(a, mode, n_pad, pdl, stream);
}

extern "C" int qd_tc_qkv_rope_append(const void* xpk, int n_pad, int m_act, const void* w_packed, int64_t k,
                                     const void* q_norm, const void* k_norm, const void* cos, const void* sin,
                                     const int64_t* pos, int64_t cap, int nq_heads, int nkv_heads, void* q_out,
                                     void* k_cache, void* v_cache, int64_t cs_b, int64_t cs_h, void* raw_out, int grid,
                                     void* scratch, int64_t scratch_bytes, int* err, int pdl, cudaStream_t stream) {
  if (nq_heads <= 0 || nkv_heads <= 0) return set_error(QD_ERR_ARG, "head counts must be positive");
  const int64_t n = (int64_t)(nq_heads + 2 * nkv_heads) * 128;
  GemvArgs a;
  if (int rc = tc_common(a, xpk, n_pad, m_act, w_packed, n, k, grid, scratch, scratch_bytes, err)) return rc;
  if (!q_norm || !k_norm || !cos || !sin || !pos || !q_out || !k_cache || !v_cache)
    return set_error(QD_ERR_ARG, "null qkv epilogue pointer");
  if (cap < 1 || cs_h < cap * 128 || cs_b < (int64_t)nkv_heads * cs_h) return set_error(QD_ERR_ARG, "cache strides");
  a.q_norm = static_cast<const __nv_bfloat16*>(q_norm);
  a.k_norm = static_cast<const __nv_bfloat16*>(k_norm);
  a.cos = static_cast<const __nv_bfloat16*>(cos);
  a.sin = static_cast<const __nv_bfloat16*>(sin);
  a.pos = pos;
  a.cap = cap;
  a.nq = nq_heads;
  a.nkv = nkv_heads;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.cs_b = cs_b;
  a.cs_h = cs_h;
  a.raw_out = static_cast<__nv_bfloat16*>(raw_out);
  return tc_launch(a, MODE_QKV, n_pad, pdl, stream);
}

extern "C" int qd_tc_lm_head_argmax(const void* xpk, int n_pad, int m_act, const void* e_packed, int64_t vocab,
                                    int64_t k, int64_t* tok, int64_t* pos, int inc_pos, void* logits_out,
                                    int64_t ld_logits, int grid, void* scratch, int64_t scratch_bytes, int* err,
                                    int pdl, cudaStream_t stream) {
  if (vocab <= 0 || vocab > 0x7fffffffLL) return set_error(QD_ERR_ARG, "vocab out of range");
  const int64_t n = (vocab + kBlockRows - 1) / kBlockRows * kBlockRows;
  GemvArgs a;
  if (int rc = tc_common(a, xpk, n_pad, m_act, e_packed, n, k, grid, scratch, scratch_bytes, err)) return rc;
  if (!tok) return set_error(QD_ERR_ARG, "null tok");
  if (inc_pos && !pos) return set_error(QD_ERR_ARG, "inc_pos needs pos");
  if (logits_out && ld_logits < vocab) return set_error(QD_ERR_ARG, "ld_logits < vocab");
  a.n_valid = vocab;
  a.tok = tok;
  a.pos_inc = pos;
  a.inc_pos = inc_pos;
  a.logits = static_cast<__nv_bfloat16*>(logits_out);
  a.ld_logits = ld_logits;
  return tc_launch(a, MODE_LM, n_pad, pdl, stream);
}

#ifdef QD_TC_TRACE
extern "C" int qd_tc_trace_set(void* p) {
  return cudaMemcpyToSymbol(qd::g_tc_trace, &p, sizeof(p)) == cudaSuccess ? 0 : 3;
}
#endif
