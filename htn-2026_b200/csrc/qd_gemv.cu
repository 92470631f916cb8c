// Streaming BF16 GEMV / skinny GEMM (m <= 8 rows) for the decode step, sm_100a.
//
// One persistent-style launch per projection. The packed weight matrix is a sequence of 16 KiB
// blocks (128 rows x 64 columns, see qd_common.cuh); the T blocks are split stream-K style into G
// contiguous ranges, one per CTA (G = one CTA per SM by default), so every CTA streams the same
// number of bytes +-1 block whatever the matrix shape. Inside a CTA a producer warp keeps a ring of
// NST blocks in flight with one-dimensional bulk copies (TMA, completion on an mbarrier); eight
// consumer warps multiply each block by the activation rows held in shared memory with fp32 FMAs,
// accumulating per (row, activation row) in registers while the block's row group stays the same.
//
// When a CTA leaves a row group it reduces its partial sums (warp shuffles) into shared memory.
// If it covered the whole group it runs the epilogue directly; otherwise it stores the partial to
// scratch and takes a ticket: the CTA whose blocks complete the group sums every partial of that
// group in fixed order (deterministic) and runs the epilogue. No spin waits between CTAs.
//
// Epilogues (all BF16 rounding points of transformers' modeling_qwen3 kept):
//   STORE, RES (residual add), SWIGLU (gate/up interleaved), QKV (per-head RMSNorm + RoPE + KV
//   append / q store), LM (logits, argmax with lowest index on ties, global argmax by the last CTA,
//   position advance).
// Prologue: the activation rows are staged in shared memory, RMSNorm-ed when a norm weight is given
// (each CTA computes the row statistics itself, so no statistics travel between kernels).
//
// Launched with programmatic dependent launch: the producer warp starts streaming weights (which no
// kernel writes) before the preceding kernel has finished; consumers wait for it before touching
// activations.

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "qd_common.cuh"
#include "qd_host.h"

namespace qd {

enum { MODE_STORE = 0, MODE_RES = 1, MODE_SWIGLU = 2, MODE_QKV = 3, MODE_LM = 4 };

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;

struct GemvArgs {
  const __nv_bfloat16* x;
  int64_t ldx;
  const char* w;
  int64_t n, n_valid, k;
  int kblocks;
  int64_t total;
  int grid, nst;
  __nv_bfloat16* out;
  int64_t ldo;
  const __nv_bfloat16* res;
  int64_t ldr;
  const __nv_bfloat16* norm_w;
  float eps;
  float* partials;
  int* tickets;
  int smax;
  int* err;
  // QKV
  const __nv_bfloat16 *q_norm, *k_norm, *cos, *sin;
  const int64_t* pos;
  int64_t cap;
  int nq, nkv;
  __nv_bfloat16 *q_out, *k_cache, *v_cache;
  int64_t cs_b, cs_h;
  __nv_bfloat16* raw_out;
  // LM
  int64_t* tok;
  int64_t* pos_inc;
  int inc_pos;
  __nv_bfloat16* logits;
  int64_t ld_logits;
  float* cta_val;
  int* cta_idx;
  int* lm_ticket;
};

struct SmemLayout {
  int ring, xs, red, wsum, lmv, lmi, flags, bars, total;
};

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline SmemLayout smem_layout(int M, int64_t k, int nst) {
  SmemLayout L;
  int off = 0;
  L.ring = off;
  off += nst * kBlockBytes;
  L.xs = off;
  off = align_up(off + (int)(M * k * 2), 128);
  L.red = off;
  off += M * kBlockRows * 4;
  L.wsum = off;
  off += M * kConsumerWarps * 4 + 64;
  L.lmv = off;
  off += 8 * 4;
  L.lmi = off;
  off += 8 * 4;
  L.flags = off;
  off += 16;
  L.bars = align_up(off, 8);
  off = L.bars + 2 * nst * 8;
  L.total = align_up(off, 128);
  return L;
}

// ------------------------------------------------------------------ epilogues (256 consumer threads)
template <int M, int MODE>
__device__ void finalize_group(const GemvArgs& a, int g, float* red, float* wsum, float* lmv, int* lmi, int tid) {
  if constexpr (MODE == MODE_STORE || MODE == MODE_RES) {
    for (int idx = tid; idx < M * kBlockRows; idx += kConsumers) {
      const int m = idx >> 7, r = idx & 127;
      const int64_t n = (int64_t)g * kBlockRows + r;
      float v = bf16r(red[idx]);
      if constexpr (MODE == MODE_RES) {
        const uint16_t rb = __ldcg(reinterpret_cast<const unsigned short*>(a.res + m * a.ldr + n));
        v = __uint_as_float((uint32_t)rb << 16) + v;
      }
      a.out[m * a.ldo + n] = __float2bfloat16_rn(v);
    }
  } else if constexpr (MODE == MODE_SWIGLU) {
    for (int idx = tid; idx < M * 64; idx += kConsumers) {
      const int m = idx >> 6, j = idx & 63;
      const float gv = bf16r(red[m * kBlockRows + j]);
      const float uv = bf16r(red[m * kBlockRows + 64 + j]);
      const float s = bf16r(gv / (1.0f + expf(-gv)));
      a.out[m * a.ldo + (int64_t)g * 64 + j] = __float2bfloat16_rn(s * uv);
    }
  } else if constexpr (MODE == MODE_QKV) {
    const int64_t p = ld_cg_s64(a.pos);
    const int warp = tid >> 5, lane = tid & 31;
    if (p < 0 || p >= a.cap) {  // never write outside the cache or read outside the RoPE tables
      if (tid == 0 && a.err) atomicOr(a.err, QD_DEVERR_POS);
      return;
    }
    // BF16 projection output
    for (int idx = tid; idx < M * kBlockRows; idx += kConsumers) {
      const float v = bf16r(red[idx]);
      red[idx] = v;
      if (a.raw_out) a.raw_out[(idx >> 7) * a.n + (int64_t)g * kBlockRows + (idx & 127)] = __float2bfloat16_rn(v);
    }
    if (g >= a.nq + a.nkv) {  // V head: append as is
      const int kvh = g - a.nq - a.nkv;
      for (int idx = tid; idx < M * kBlockRows; idx += kConsumers) {
        const int m = idx >> 7, r = idx & 127;
        a.v_cache[m * a.cs_b + kvh * a.cs_h + p * 128 + r] = __float2bfloat16_rn(red[idx]);
      }
      return;
    }
    // per-head RMSNorm (Qwen3RMSNorm over 128): sum of squares per activation row
    for (int base = 0; base < M * kBlockRows; base += kConsumers) {
      const int idx = base + tid;
      float sq = 0.f;
      if (idx < M * kBlockRows) sq = red[idx] * red[idx];
      sq = warp_sum(sq);
      if (lane == 0 && idx < M * kBlockRows) wsum[idx >> 5] = sq;  // one slot per 32 rows
    }
    named_bar(1, kConsumers);
    const __nv_bfloat16* nw = (g < a.nq) ? a.q_norm : a.k_norm;
    for (int idx = tid; idx < M * kBlockRows; idx += kConsumers) {
      const int m = idx >> 7, r = idx & 127;
      const float var = (wsum[m * 4 + 0] + wsum[m * 4 + 1] + wsum[m * 4 + 2] + wsum[m * 4 + 3]) / 128.0f;
      const float rstd = 1.0f / sqrtf(var + a.eps);
      const float y = bf16r(bf16_to_f(nw[r]) * bf16r(red[idx] * rstd));
      red[idx] = y;  // each thread rewrites only its own entries; partners are read after the barrier
    }
    named_bar(1, kConsumers);
    for (int idx = tid; idx < M * kBlockRows; idx += kConsumers) {
      const int m = idx >> 7, r = idx & 127;
      const float y = red[idx];
      const float yp = red[(idx & ~127) | (r ^ 64)];
      const float c = bf16_to_f(a.cos[p * 128 + r]);
      const float s = bf16_to_f(a.sin[p * 128 + r]);
      // q*cos + rotate_half(q)*sin with every product a BF16 tensor (rotate_half = cat(-q2, q1))
      const float rot = (r < 64) ? bf16r(-yp * s) : bf16r(yp * s);
      const __nv_bfloat16 o = __float2bfloat16_rn(bf16r(y * c) + rot);
      if (g < a.nq) {
        a.q_out[((int64_t)m * a.nq + g) * 128 + r] = o;
      } else {
        a.k_cache[m * a.cs_b + (g - a.nq) * a.cs_h + p * 128 + r] = o;
      }
    }
    (void)warp;
  } else if constexpr (MODE == MODE_LM) {
    const int warp = tid >> 5, lane = tid & 31;
    for (int base = 0; base < M * kBlockRows; base += kConsumers) {
      const int idx = base + tid;
      float v = -INFINITY;
      int n = 0x7fffffff;
      if (idx < M * kBlockRows) {
        const int m = idx >> 7, r = idx & 127;
        const int64_t row = (int64_t)g * kBlockRows + r;
        if (row < a.n_valid) {
          v = bf16r(red[idx]);
          n = (int)row;
          if (a.logits) a.logits[m * a.ld_logits + row] = __float2bfloat16_rn(v);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int on = __shfl_xor_sync(0xffffffffu, n, o);
        if (ov > v || (ov == v && on < n)) {
          v = ov;
          n = on;
        }
      }
      if (lane == 0 && idx < M * kBlockRows) {
        wsum[(idx >> 5) * 2] = v;
        reinterpret_cast<int*>(wsum)[(idx >> 5) * 2 + 1] = n;
      }
    }
    named_bar(1, kConsumers);
    if (tid < M) {
      float bv = lmv[tid];
      int bi = lmi[tid];
      for (int q = 0; q < 4; ++q) {
        const float v = wsum[(tid * 4 + q) * 2];
        const int n = reinterpret_cast<int*>(wsum)[(tid * 4 + q) * 2 + 1];
        if (v > bv || (v == bv && n < bi)) {
          bv = v;
          bi = n;
        }
      }
      lmv[tid] = bv;
      lmi[tid] = bi;
    }
    (void)warp;
  }
}

template <int M, int MODE>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(1024) char smem[];
  const SmemLayout L = smem_layout(M, a.k, a.nst);
  char* ring = smem + L.ring;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + L.xs);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* wsum = reinterpret_cast<float*>(smem + L.wsum);
  float* lmv = reinterpret_cast<float*>(smem + L.lmv);
  int* lmi = reinterpret_cast<int*>(smem + L.lmi);
  int* flags = reinterpret_cast<int*>(smem + L.flags);
  const uint32_t bars = smem_u32(smem + L.bars);
  const int nst = a.nst;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (nst + s); };

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  const int64_t b_begin = part_begin(a.total, a.grid, cta);
  const int64_t b_end = part_begin(a.total, a.grid, cta + 1);
  const int nblk = (int)(b_end - b_begin);

  if (tid == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), kConsumerWarps);
    }
    fence_mbar_init();
    flags[0] = 0;  // blocks issued by the producer
    flags[1] = 0;  // ticket result broadcast
  }
  if (tid < M) {
    lmv[tid] = -INFINITY;
    lmi[tid] = 0x7fffffff;
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer warp
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int issued = 0;
      for (int it = 0; it < nblk; ++it) {
        const int s = it % nst;
        const int round = it / nst;
        if (round > 0 && !mbar_wait(empty_bar(s), (round - 1) & 1, a.err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(full_bar(s), kBlockBytes);
        bulk_g2s(smem_u32(ring + s * kBlockBytes), a.w + (b_begin + it) * (int64_t)kBlockBytes, kBlockBytes,
                 full_bar(s), pol);
        issued = it + 1;
      }
      flags[0] = issued;
    }
  } else {
    // ------------------------------------------------------------ consumers
    grid_dep_wait();
    grid_dep_launch();
    // stage activations (and RMSNorm them) in shared memory
    const int kv8 = (int)(a.k >> 3);
    for (int m = 0; m < M; ++m) {
      float sq = 0.f;
      for (int q = tid; q < kv8; q += kConsumers) {
        const uint4 v = ld_cg_v4(a.x + m * a.ldx + q * 8);
        *reinterpret_cast<uint4*>(xs + (int64_t)m * a.k + q * 8) = v;
        if (a.norm_w) {
          const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = bf_lo(u[e]), hi = bf_hi(u[e]);
            sq = fmaf(lo, lo, sq);
            sq = fmaf(hi, hi, sq);
          }
        }
      }
      if (a.norm_w) {
        sq = warp_sum(sq);
        if (lane == 0) wsum[m * kConsumerWarps + warp] = sq;
      }
    }
    named_bar(1, kConsumers);
    if (a.norm_w) {
      // Qwen3RMSNorm: w * bf16(x * rsqrt(mean(x^2) + eps)), rounded to BF16
      for (int m = 0; m < M; ++m) {
        float ss = 0.f;
#pragma unroll
        for (int w8 = 0; w8 < kConsumerWarps; ++w8) ss += wsum[m * kConsumerWarps + w8];
        const float rstd = 1.0f / sqrtf(ss / (float)a.k + a.eps);
        for (int q = tid; q < kv8; q += kConsumers) {
          uint4* p = reinterpret_cast<uint4*>(xs + (int64_t)m * a.k + q * 8);
          const uint4 xv = *p;
          const uint4 wv = *reinterpret_cast<const uint4*>(a.norm_w + q * 8);
          const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w};
          const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = bf16r(bf_lo(wu[e]) * bf16r(bf_lo(xu[e]) * rstd));
            const float hi = bf16r(bf_hi(wu[e]) * bf16r(bf_hi(xu[e]) * rstd));
            o[e] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
          }
          *p = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      named_bar(1, kConsumers);
    }

    // per-lane geometry inside a 128x64 block
    const int rsub = lane >> 3;  // 0..3
    const int c = lane & 7;      // logical 16-byte chunk (8 columns)
    int roff[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 16 * warp + rsub + 4 * i;
      roff[i] = r * 128 + ((c ^ (r & 7)) << 4);
    }

    float acc[4][M];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[i][m] = 0.f;

    bool ok = true;
    int64_t seg_first = b_begin;  // first block of the current segment
    int g = (int)(b_begin / a.kblocks);
    int kb = (int)(b_begin - (int64_t)g * a.kblocks) - 1;
    int s = -1, phase = 0;
    for (int it = 0; it < nblk; ++it) {
      const int64_t b = b_begin + it;
      if (++kb == a.kblocks) {
        kb = 0;
        ++g;
      }
      if (++s == nst) {
        s = 0;
        phase ^= 1;
      }
      if (ok) ok = mbar_wait(full_bar(s), phase, a.err, kErrWaitFull);
      {
        const char* blk = ring + s * kBlockBytes;
        float xv[M][8];
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const uint4 u = *reinterpret_cast<const uint4*>(xs + (int64_t)m * a.k + kb * 64 + c * 8);
          xv[m][0] = bf_lo(u.x);
          xv[m][1] = bf_hi(u.x);
          xv[m][2] = bf_lo(u.y);
          xv[m][3] = bf_hi(u.y);
          xv[m][4] = bf_lo(u.z);
          xv[m][5] = bf_hi(u.z);
          xv[m][6] = bf_lo(u.w);
          xv[m][7] = bf_hi(u.w);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 u = *reinterpret_cast<const uint4*>(blk + roff[i]);
          const float w8[8] = {bf_lo(u.x), bf_hi(u.x), bf_lo(u.y), bf_hi(u.y),
                               bf_lo(u.z), bf_hi(u.z), bf_lo(u.w), bf_hi(u.w)};
#pragma unroll
          for (int m = 0; m < M; ++m)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[i][m] = fmaf(w8[e], xv[m][e], acc[i][m]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(s));

      const bool seg_end = (kb == a.kblocks - 1) || (it == nblk - 1);
      if (!seg_end) continue;

      // ---------------------------------------------------------- flush the segment of group g
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int m = 0; m < M; ++m) {
          float v = acc[i][m];
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          acc[i][m] = 0.f;
          if (c == 0) red[m * kBlockRows + 16 * warp + rsub + 4 * i] = v;
        }
      named_bar(1, kConsumers);
      const int64_t gb0 = (int64_t)g * a.kblocks;
      const int nseg_blk = (int)(b + 1 - seg_first);
      if (seg_first == gb0 && nseg_blk == a.kblocks) {
        finalize_group<M, MODE>(a, g, red, wsum, lmv, lmi, tid);
      } else {
        const int c_lo = part_owner(a.total, a.grid, gb0);
        float* dst = a.partials + ((int64_t)g * a.smax + (cta - c_lo)) * (M * kBlockRows);
        for (int idx = tid; idx < M * kBlockRows; idx += kConsumers) dst[idx] = red[idx];
        __threadfence();
        named_bar(1, kConsumers);
        if (tid == 0) {
          const int old = atomicAdd(a.tickets + g, nseg_blk);
          flags[1] = (old + nseg_blk == a.kblocks) ? 1 : 0;
        }
        named_bar(1, kConsumers);
        if (flags[1]) {
          __threadfence();
          const int c_hi = part_owner(a.total, a.grid, gb0 + a.kblocks - 1);
          for (int idx = tid; idx < M * kBlockRows; idx += kConsumers) {
            float sum = 0.f;
            for (int cc = c_lo; cc <= c_hi; ++cc) {
              const int64_t s0 = part_begin(a.total, a.grid, cc), s1 = part_begin(a.total, a.grid, cc + 1);
              if ((s1 < gb0 + a.kblocks ? s1 : gb0 + a.kblocks) <= (s0 > gb0 ? s0 : gb0)) continue;
              sum += ld_cg_f32(a.partials + ((int64_t)g * a.smax + (cc - c_lo)) * (M * kBlockRows) + idx);
            }
            red[idx] = sum;
          }
          named_bar(1, kConsumers);
          finalize_group<M, MODE>(a, g, red, wsum, lmv, lmi, tid);
          if (tid == 0) atomicExch(a.tickets + g, 0);
        }
      }
      named_bar(1, kConsumers);
      seg_first = b + 1;
    }

    if constexpr (MODE == MODE_LM) {
      // global argmax: every CTA posts its best per row; the last CTA reduces them in full
      if (tid < M) {
        a.cta_val[tid * a.grid + cta] = lmv[tid];
        a.cta_idx[tid * a.grid + cta] = lmi[tid];
      }
      __threadfence();
      named_bar(1, kConsumers);
      if (tid == 0) flags[1] = (atomicAdd(a.lm_ticket, 1) == a.grid - 1) ? 1 : 0;
      named_bar(1, kConsumers);
      if (flags[1]) {
        __threadfence();
        for (int m = 0; m < M; ++m) {
          float bv = -INFINITY;
          int bi = 0x7fffffff;
          for (int q = tid; q < a.grid; q += kConsumers) {
            const float v = ld_cg_f32(a.cta_val + m * a.grid + q);
            const int n = (int)__ldcg(a.cta_idx + m * a.grid + q);
            if (v > bv || (v == bv && n < bi)) {
              bv = v;
              bi = n;
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int on = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && on < bi)) {
              bv = ov;
              bi = on;
            }
          }
          if (lane == 0) {
            wsum[warp * 2] = bv;
            reinterpret_cast<int*>(wsum)[warp * 2 + 1] = bi;
          }
          named_bar(1, kConsumers);
          if (tid == 0) {
            for (int w8 = 1; w8 < kConsumerWarps; ++w8) {
              const float v = wsum[w8 * 2];
              const int n = reinterpret_cast<int*>(wsum)[w8 * 2 + 1];
              if (v > bv || (v == bv && n < bi)) {
                bv = v;
                bi = n;
              }
            }
            a.tok[m] = (int64_t)bi;
          }
          named_bar(1, kConsumers);
        }
        if (tid == 0) {
          if (a.inc_pos && a.pos_inc) a.pos_inc[0] = a.pos_inc[0] + 1;
          atomicExch(a.lm_ticket, 0);
        }
      }
    }
    (void)ok;
  }

  __syncthreads();
  // drain: never exit with a bulk copy still writing this CTA's shared memory
  if (tid == 0) {
    const int issued = flags[0];
    for (int it = issued > nst ? issued - nst : 0; it < issued; ++it)
      if (!mbar_wait(full_bar(it % nst), (it / nst) & 1, a.err, kErrDrain)) break;
  }
}

// ------------------------------------------------------------------ host side
struct Plan {
  int grid, smax, nst;
  int64_t groups, total;
  int64_t off_tickets, off_lm_ticket, off_cta_val, off_cta_idx, off_partials, bytes;
};

static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

// Tuning: QD_GEMV_CTAS_PER_SM CTAs per SM in the grid (default 1), QD_GEMV_STAGES ring depth in 16 KiB
// blocks (default 4), reduced until the CTA's shared memory fits its share of the SM.
static int ctas_per_sm() {
  const int c = env_int("QD_GEMV_CTAS_PER_SM", 1);
  return c < 1 ? 1 : (c > 4 ? 4 : c);
}

static int default_nst(int M, int64_t k) {
  const int fixed = smem_layout(M, k, 0).total;
  const int budget = (ctas_per_sm() == 1 ? 227 * 1024 : 228 * 1024 / ctas_per_sm() - 1024);
  int nst = env_int("QD_GEMV_STAGES", 4);
  if (nst > 16) nst = 16;
  while (nst > 2 && fixed + nst * kBlockBytes + 16 * nst > budget) --nst;
  return nst < 2 ? 2 : nst;
}

static bool make_plan(int64_t n_rows, int64_t k, int M, int grid_hint, Plan* p) {
  if (n_rows <= 0 || k <= 0 || n_rows % kBlockRows || k % kBlockCols || M < 1 || M > 8) return false;
  const int kblocks = (int)(k / kBlockCols);
  p->groups = n_rows / kBlockRows;
  p->total = p->groups * kblocks;
  int g = grid_hint > 0 ? grid_hint : host_sm_count() * ctas_per_sm();
  if (g > p->total) g = (int)p->total;
  if (g < 1) g = 1;
  p->grid = g;
  int smax = 1;
  for (int64_t gi = 0; gi < p->groups; ++gi) {
    const int lo = part_owner(p->total, g, gi * kblocks), hi = part_owner(p->total, g, gi * kblocks + kblocks - 1);
    if (hi - lo + 1 > smax) smax = hi - lo + 1;
  }
  p->smax = smax;
  p->nst = default_nst(M, k);
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  p->off_tickets = take(p->groups * 4);
  p->off_lm_ticket = take(4);
  p->off_cta_val = take((int64_t)M * g * 4);
  p->off_cta_idx = take((int64_t)M * g * 4);
  p->off_partials = take(p->groups * smax * M * kBlockRows * 4);
  p->bytes = off;
  return true;
}

template <int M, int MODE>
static int launch_m(const GemvArgs& a, int smem, int pdl, cudaStream_t stream) {
  auto kern = gemv_kernel<M, MODE>;
  static int configured = 0;
  if (smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return set_error(QD_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured = smem;
  }
  return launch_kernel((const void*)kern, dim3(a.grid), dim3(kThreads), smem, pdl, stream, (void*)&a);
}

template <int MODE>
static int launch_mode(const GemvArgs& a, int M, int smem, int pdl, cudaStream_t stream) {
  switch (M) {
    case 1: return launch_m<1, MODE>(a, smem, pdl, stream);
    case 2: return launch_m<2, MODE>(a, smem, pdl, stream);
    case 3: return launch_m<3, MODE>(a, smem, pdl, stream);
    case 4: return launch_m<4, MODE>(a, smem, pdl, stream);
    case 5: return launch_m<5, MODE>(a, smem, pdl, stream);
    case 6: return launch_m<6, MODE>(a, smem, pdl, stream);
    case 7: return launch_m<7, MODE>(a, smem, pdl, stream);
    case 8: return launch_m<8, MODE>(a, smem, pdl, stream);
  }
  return set_error(QD_ERR_UNSUPPORTED, "m=%d outside 1..8", M);
}

static int launch_any(const GemvArgs& a, int mode, int M, int pdl, cudaStream_t stream) {
  const int smem = smem_layout(M, a.k, a.nst).total;
  if (smem > 227 * 1024) return set_error(QD_ERR_UNSUPPORTED, "shared memory %d B exceeds 227 KiB (m=%d k=%lld)",
                                          smem, M, (long long)a.k);
  switch (mode) {
    case MODE_STORE: return launch_mode<MODE_STORE>(a, M, smem, pdl, stream);
    case MODE_RES: return launch_mode<MODE_RES>(a, M, smem, pdl, stream);
    case MODE_SWIGLU: return launch_mode<MODE_SWIGLU>(a, M, smem, pdl, stream);
    case MODE_QKV: return launch_mode<MODE_QKV>(a, M, smem, pdl, stream);
    case MODE_LM: return launch_mode<MODE_LM>(a, M, smem, pdl, stream);
  }
  return set_error(QD_ERR_ARG, "unknown epilogue %d", mode);
}

static bool fill_common(GemvArgs& a, const Plan& p, const void* x, int64_t ldx, const void* w, int64_t n_rows,
                        int64_t k, int M, const void* norm_w, float eps, void* scratch) {
  a = GemvArgs{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.w = static_cast<const char*>(w);
  a.n = n_rows;
  a.n_valid = n_rows;
  a.k = k;
  a.kblocks = (int)(k / kBlockCols);
  a.total = p.total;
  a.grid = p.grid;
  a.nst = p.nst;
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  char* sc = static_cast<char*>(scratch);
  a.tickets = reinterpret_cast<int*>(sc + p.off_tickets);
  a.lm_ticket = reinterpret_cast<int*>(sc + p.off_lm_ticket);
  a.cta_val = reinterpret_cast<float*>(sc + p.off_cta_val);
  a.cta_idx = reinterpret_cast<int*>(sc + p.off_cta_idx);
  a.partials = reinterpret_cast<float*>(sc + p.off_partials);
  a.smax = p.smax;
  (void)M;
  return true;
}

static int check_x(const void* x, int64_t ldx, int64_t k, const void* w, const void* norm_w) {
  if (!x || !w) return set_error(QD_ERR_ARG, "null x or weight pointer");
  if (!aligned16(x) || !aligned16(w) || ldx < k || ldx % 8) return set_error(QD_ERR_ARG, "x/w must be 16-byte aligned, ldx >= k and a multiple of 8");
  if (norm_w && !aligned16(norm_w)) return set_error(QD_ERR_ARG, "norm weight must be 16-byte aligned");
  return QD_OK;
}

}  // namespace qd

using namespace qd;

extern "C" int qd_gemv_plan(int64_t n, int64_t k, int m, int grid_hint, int* grid, int64_t* scratch_bytes) {
  Plan p;
  if (!make_plan(n, k, m, grid_hint, &p))
    return set_error(QD_ERR_UNSUPPORTED, "gemv plan: n=%lld k=%lld m=%d (need n%%128==0, k%%64==0, 1<=m<=8)",
                     (long long)n, (long long)k, m);
  if (grid) *grid = p.grid;
  if (scratch_bytes) *scratch_bytes = p.bytes;
  return QD_OK;
}

extern "C" int qd_lm_head_plan(int64_t vocab, int64_t k, int m, int grid_hint, int* grid, int64_t* scratch_bytes) {
  return qd_gemv_plan((vocab + kBlockRows - 1) / kBlockRows * kBlockRows, k, m, grid_hint, grid, scratch_bytes);
}

extern "C" int qd_gemv(const void* x, int64_t ldx, const void* w_packed, int64_t n, int64_t k, int m, void* out,
                       int64_t ldo, const void* res, int64_t ldr, const void* norm_w, float eps, int epilogue,
                       int grid, void* scratch, int64_t scratch_bytes, int* err, int pdl, cudaStream_t stream) {
  Plan p;
  if (!make_plan(n, k, m, grid, &p)) return qd_gemv_plan(n, k, m, grid, nullptr, nullptr);
  if (p.grid != grid) return set_error(QD_ERR_ARG, "grid %d does not match the plan (%d)", grid, p.grid);
  if (!scratch || scratch_bytes < p.bytes)
    return set_error(QD_ERR_SCRATCH, "scratch %lld B < %lld B", (long long)scratch_bytes, (long long)p.bytes);
  if (int rc = check_x(x, ldx, k, w_packed, norm_w)) return rc;
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
  } else {
    return set_error(QD_ERR_ARG, "unknown epilogue %d", epilogue);
  }
  GemvArgs a;
  fill_common(a, p, x, ldx, w_packed, n, k, m, norm_w, eps, scratch);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.res = static_cast<const __nv_bfloat16*>(res);
  a.ldr = ldr;
  a.err = err;
  return launch_any(a, mode, m, pdl, stream);
}

extern "C" int qd_qkv_rope_append(const void* x, int64_t ldx, const void* w_packed, int64_t k, int m,
                                  const void* norm_w, float eps, const void* q_norm, const void* k_norm,
                                  const void* cos, const void* sin, const int64_t* pos, int64_t cap, int nq_heads,
                                  int nkv_heads, void* q_out, void* k_cache, void* v_cache, int64_t cs_b, int64_t cs_h,
                                  void* raw_out, int grid, void* scratch, int64_t scratch_bytes, int* err, int pdl,
                                  cudaStream_t stream) {
  const int64_t n = (int64_t)(nq_heads + 2 * nkv_heads) * 128;
  Plan p;
  if (nq_heads <= 0 || nkv_heads <= 0) return set_error(QD_ERR_ARG, "head counts must be positive");
  if (!make_plan(n, k, m, grid, &p)) return qd_gemv_plan(n, k, m, grid, nullptr, nullptr);
  if (p.grid != grid) return set_error(QD_ERR_ARG, "grid %d does not match the plan (%d)", grid, p.grid);
  if (!scratch || scratch_bytes < p.bytes)
    return set_error(QD_ERR_SCRATCH, "scratch %lld B < %lld B", (long long)scratch_bytes, (long long)p.bytes);
  if (int rc = check_x(x, ldx, k, w_packed, norm_w)) return rc;
  if (!q_norm || !k_norm || !cos || !sin || !pos || !q_out || !k_cache || !v_cache)
    return set_error(QD_ERR_ARG, "null qkv epilogue pointer");
  if (cap < 1 || cs_h < cap * 128 || cs_b < (int64_t)nkv_heads * cs_h)
    return set_error(QD_ERR_ARG, "cache capacity/strides");
  GemvArgs a;
  fill_common(a, p, x, ldx, w_packed, n, k, m, norm_w, eps, scratch);
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
  a.err = err;
  return launch_any(a, MODE_QKV, m, pdl, stream);
}

extern "C" int qd_lm_head_argmax(const void* x, int64_t ldx, const void* e_packed, int64_t vocab, int64_t k, int m,
                                 const void* norm_w, float eps, int64_t* tok, int64_t* pos, int inc_pos,
                                 void* logits_out, int64_t ld_logits, int grid, void* scratch, int64_t scratch_bytes,
                                 int* err, int pdl, cudaStream_t stream) {
  const int64_t n = (vocab + kBlockRows - 1) / kBlockRows * kBlockRows;
  Plan p;
  if (vocab <= 0 || vocab > 0x7fffffffLL) return set_error(QD_ERR_ARG, "vocab out of range");
  if (!make_plan(n, k, m, grid, &p)) return qd_gemv_plan(n, k, m, grid, nullptr, nullptr);
  if (p.grid != grid) return set_error(QD_ERR_ARG, "grid %d does not match the plan (%d)", grid, p.grid);
  if (!scratch || scratch_bytes < p.bytes)
    return set_error(QD_ERR_SCRATCH, "scratch %lld B < %lld B", (long long)scratch_bytes, (long long)p.bytes);
  if (int rc = check_x(x, ldx, k, e_packed, norm_w)) return rc;
  if (!tok) return set_error(QD_ERR_ARG, "null tok");
  if (inc_pos && !pos) return set_error(QD_ERR_ARG, "inc_pos needs pos");
  if (logits_out && ld_logits < vocab) return set_error(QD_ERR_ARG, "ld_logits < vocab");
  GemvArgs a;
  fill_common(a, p, x, ldx, e_packed, n, k, m, norm_w, eps, scratch);
  a.n_valid = vocab;
  a.tok = tok;
  a.pos_inc = pos;
  a.inc_pos = inc_pos;
  a.logits = static_cast<__nv_bfloat16*>(logits_out);
  a.ld_logits = ld_logits;
  a.err = err;
  return launch_any(a, MODE_LM, m, pdl, stream);
}

// ------------------------------------------------------------------ allocation-free entry point
// Some callers cannot hand this library a scratch buffer: a host application whose device memory is
// owned end to end by its own pool allocator and which passes only input and output buffers, a
// plugin loaded into such a host with no allocator handle of its own, or a latency-critical loop
// that must not call cudaMalloc (cudaMalloc can synchronize the device and stall other streams).
// qd_gemv_noalloc serves them: its scratch (tickets and split-K partial sums) is this file-scope
// device array, which every GPU that loads the library holds until the process exits.
namespace qd {

constexpr int64_t kNoAllocScratchBytes = 4ll << 20;  // 4 MiB: every decode projection at m <= 8
static __device__ __align__(256) char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device. In host code the array's name is only a
// host-side stand-in, so the address is looked up once per device with that device current (the
// first call on each device) and cached.
static int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(QD_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(QD_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(QD_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return QD_OK;
}

}  // namespace qd

extern "C" int qd_gemv_noalloc(const void* x, int64_t ldx, const void* w_packed, int64_t n, int64_t k, int m,
                               void* out, int64_t ldo, const void* res, int64_t ldr, const void* norm_w, float eps,
                               int epilogue, int* err, int pdl, cudaStream_t stream) {
  Plan p;
  if (!make_plan(n, k, m, 0, &p)) return qd_gemv_plan(n, k, m, 0, nullptr, nullptr);
  if (p.bytes > kNoAllocScratchBytes)
    return set_error(QD_ERR_UNSUPPORTED,
                     "qd_gemv_noalloc: n=%lld k=%lld m=%d needs %lld B of scratch, above its fixed %lld B",
                     (long long)n, (long long)k, m, (long long)p.bytes, (long long)kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // The array keeps the previous call's contents (possibly of another shape): clear the tickets and
  // the per-CTA argmax slots, everything in front of the partial sums, before this call uses them.
  cudaError_t e = cudaMemsetAsync(scratch, 0, (size_t)p.off_partials, stream);
  if (e != cudaSuccess) return set_error(QD_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  return qd_gemv(x, ldx, w_packed, n, k, m, out, ldo, res, ldr, norm_w, eps, epilogue, p.grid, scratch,
                 kNoAllocScratchBytes, err, pdl, stream);
}
