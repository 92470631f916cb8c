// Device side of the streaming GEMV, shared by the per-projection kernel (qd_gemv.cu) and the
// persistent decode-step kernel (qd_step.cu).
//
// A projection's packed weight matrix is a sequence of 16 KiB blocks (128 rows x 64 columns, see
// qd_common.cuh). Its T blocks are split stream-K into G contiguous ranges, one per CTA, so every
// CTA streams the same bytes +-1 block whatever the matrix shape. A producer warp keeps a ring of
// blocks in flight with one-dimensional bulk copies (TMA, completion on an mbarrier); eight consumer
// warps multiply each block by the activation rows staged in shared memory with fp32 FMAs and
// accumulate per (row, activation row) in registers while the block's row group stays the same.
//
// Leaving a row group, a CTA reduces its partial sums (warp shuffles) into shared memory. If it
// covered the whole group it runs the epilogue directly; otherwise it stores the partial to scratch
// and takes a ticket: the CTA whose blocks complete the group sums every partial of that group in
// fixed order (deterministic for a fixed grid) and runs the epilogue. No CTA waits on another here.
//
// Epilogues keep every BF16 rounding point of transformers' modeling_qwen3:
//   STORE   out = bf16(y)
//   RES     out = bf16(res + bf16(y))                      (residual add, may be in place)
//   SWIGLU  out = bf16(bf16(silu(bf16 g)) * bf16 u)        (gate/up interleaved per 128-row group)
//   QKV     per-head RMSNorm + RoPE (BF16 products), q store, K/V append at the device position
//   LM      BF16 logits, argmax with the lowest index on ties, folded into a per-CTA best
#pragma once

#include "qd_common.cuh"
#include "qd_host.h"

namespace qd {

enum { MODE_STORE = 0, MODE_RES = 1, MODE_SWIGLU = 2, MODE_QKV = 3, MODE_LM = 4 };

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + one producer warp
constexpr int kBarConsumers = 1;           // named barrier of the 256 consumer threads
constexpr int kStageBatch = 5;             // activation chunks per thread in flight (k <= 10240 in one pass)
constexpr int kFxStage = 1;                // stage_x_fx: chunks per thread in flight
constexpr int kNormPre = 2;                // RMSNorm weight chunks per thread preloaded (k <= 4096); more are
                                           // loaded in the normalising pass

struct GemvArgs {
  const __nv_bfloat16* x;
  int64_t ldx;
  const char* x_packed;  // tensor-core path: activations packed as [k/64][N][64] swizzled tiles
  const char* w;
  int64_t n, n_valid, k;
  int kblocks;
  int64_t total;
  int grid, nst, prefetch;
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
  int m_act;       // activation rows that are real (<= M; the tensor-core path pads M to 16s)
  int out_npad;    // SWIGLU: 0 = row-major out; else out is the next projection's packed operand
  int* done;       // optional: +1 (release) per finalized row group
  // RES and QKV epilogues with fixed-point group sums (CUDA-core kernels): a row group's total is
  // fx_to_float(sum over its segments of fx_of(partial)), an exact integer sum and so independent of the
  // order the partials are added in. fx_numerics alone: the last arriver sums the stored partials that
  // way. fx (persistent step): no CTA finalizes - every segment adds its rows into fx ([m][n] int64)
  // with integer atomics and its K-block count into *fx_ctr (release), and the next op's staging applies
  // the epilogue from the sums itself.
  int fx_numerics;
  int64_t* fx;
  int* fx_ctr;
  int pos_ready;   // QKV: flags[2] already holds the position and aux its cos/sin rows
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

// Fixed-point partial sums: value * 2^32 rounded to int64 (exact for |value| < 2^31 at a resolution of
// 2^-32, far below a BF16 output's rounding), added with integer atomics (associative, so the sum does
// not depend on the order of the contributions) and converted back with one rounding to fp32.
__device__ __forceinline__ long long fx_of(float v) { return __float2ll_rn(v * 4294967296.0f); }
__device__ __forceinline__ float fx_to_float(long long s) { return __ll2float_rn(s) * 2.3283064365386963e-10f; }

// Ring of 16 KiB blocks in shared memory with a full and an empty mbarrier per slot.
struct Ring {
  char* base;
  uint32_t bars;
  int nst;
  __device__ __forceinline__ uint32_t full(int s) const { return bars + 8u * s; }
  __device__ __forceinline__ uint32_t empty(int s) const { return bars + 8u * (nst + s); }
};

__device__ __forceinline__ void ring_init(const Ring& R) {
  for (int s = 0; s < R.nst; ++s) {
    mbar_init(R.full(s), 1);
    mbar_init(R.empty(s), kConsumerWarps);
  }
  fence_mbar_init();
}

// Producer (one lane): issue `nblk` consecutive blocks starting at `src`. slot / round carry across
// calls so several projections can share one ring. Returns false if a wait for a free slot expired.
__device__ __forceinline__ bool produce_blocks(const Ring& R, int& slot, int& round, int& issued, const char* src,
                                               int64_t nblk, uint64_t pol, int* err) {
  for (int64_t i = 0; i < nblk; ++i) {
    if (round > 0 && !mbar_wait(R.empty(slot), (round - 1) & 1, err, kErrWaitEmpty)) return false;
    mbar_arrive_expect_tx(R.full(slot), kBlockBytes);
    bulk_g2s(smem_u32(R.base + slot * kBlockBytes), src + i * (int64_t)kBlockBytes, kBlockBytes, R.full(slot), pol);
    ++issued;
    if (++slot == R.nst) {
      slot = 0;
      ++round;
    }
  }
  return true;
}

// Producer over one contiguous range of blocks with an L2 lookahead: before waiting for a free ring
// slot it keeps `ahead` blocks beyond the next issue prefetched into L2, so HBM keeps streaming while
// the ring is full (the later bulk copies then hit L2).
__device__ __forceinline__ bool produce_range_prefetch(const Ring& R, int& slot, int& round, int& issued,
                                                       const char* src, int64_t nblk, int ahead, uint64_t pol,
                                                       int* err) {
  int64_t pf = 0;
  for (int64_t i = 0; i < nblk; ++i) {
    for (; pf < nblk && pf <= i + ahead; ++pf) prefetch_l2(src + pf * (int64_t)kBlockBytes, kBlockBytes);
    if (round > 0 && !mbar_wait(R.empty(slot), (round - 1) & 1, err, kErrWaitEmpty)) return false;
    mbar_arrive_expect_tx(R.full(slot), kBlockBytes);
    bulk_g2s(smem_u32(R.base + slot * kBlockBytes), src + i * (int64_t)kBlockBytes, kBlockBytes, R.full(slot), pol);
    ++issued;
    if (++slot == R.nst) {
      slot = 0;
      ++round;
    }
  }
  return true;
}

// Never leave with a bulk copy still writing shared memory: wait (bounded) for the last `nst`
// issued blocks. Call from one thread after every consumer is done.
__device__ __forceinline__ void ring_drain(const Ring& R, int issued, int* err) {
  for (int it = issued > R.nst ? issued - R.nst : 0; it < issued; ++it)
    if (!mbar_wait(R.full(it % R.nst), (it / R.nst) & 1, err, kErrDrain)) break;
}

__device__ __forceinline__ void signal_done(int* done, int tid) {
  fence_proxy_async_global();  // results this CTA wrote may be read next by another CTA's bulk copies
  named_bar(kBarConsumers, kConsumers);
  if (tid == 0) red_release_add(done, 1);
}

// Stage the activation rows x[0..M) in shared memory, RMSNorm-ed when a.norm_w is set:
// xs = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))) (Qwen3RMSNorm's cast placement). 256 threads.
template <int M>
__device__ void stage_x(const GemvArgs& a, __nv_bfloat16* xs, float* wsum, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int kv8 = (int)(a.k >> 3);
  // the first norm weights this thread applies, loaded with its first activation row
  uint4 nwv[kNormPre];
  if (a.norm_w) {
#pragma unroll
    for (int j = 0; j < kNormPre; ++j) {
      const int q = j * kConsumers + tid;
      nwv[j] = q < kv8 ? *reinterpret_cast<const uint4*>(a.norm_w + q * 8) : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  for (int m = 0; m < M; ++m) {
    float sq = 0.f;
    for (int q0 = 0; q0 < kv8; q0 += kStageBatch * kConsumers) {
      uint4 v[kStageBatch];  // all of this thread's loads in flight before the first is used
#pragma unroll
      for (int j = 0; j < kStageBatch; ++j) {
        const int q = q0 + j * kConsumers + tid;
        v[j] = q < kv8 ? ld_cg_v4(a.x + m * a.ldx + q * 8) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int j = 0; j < kStageBatch; ++j) {
        const int q = q0 + j * kConsumers + tid;
        if (q >= kv8) continue;
        *reinterpret_cast<uint4*>(xs + (int64_t)m * a.k + q * 8) = v[j];
        if (a.norm_w) {
          const uint32_t u[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = bf_lo(u[e]), hi = bf_hi(u[e]);
            sq = fmaf(lo, lo, sq);
            sq = fmaf(hi, hi, sq);
          }
        }
      }
    }
    if (a.norm_w) {
      sq = warp_sum(sq);
      if (lane == 0) wsum[m * kConsumerWarps + warp] = sq;
    }
  }
  named_bar(kBarConsumers, kConsumers);
  if (a.norm_w) {
    for (int m = 0; m < M; ++m) {
      float ss = 0.f;
#pragma unroll
      for (int w8 = 0; w8 < kConsumerWarps; ++w8) ss += wsum[m * kConsumerWarps + w8];
      const float rstd = 1.0f / sqrtf(ss / (float)a.k + a.eps);
      // xs chunk q (8 values) <- bf16(w * bf16(x * rstd)), w the norm weights of chunk q
      auto norm_chunk = [&](int q, const uint4 wv) {
        uint4* p = reinterpret_cast<uint4*>(xs + (int64_t)m * a.k + q * 8);
        const uint4 xv = *p;
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
      };
#pragma unroll
      for (int j = 0; j < kNormPre; ++j)  // preloaded weights (constant indices: they stay in registers)
        if (j * kConsumers + tid < kv8) norm_chunk(j * kConsumers + tid, nwv[j]);
      for (int q = kNormPre * kConsumers + tid; q < kv8; q += kConsumers)
        norm_chunk(q, *reinterpret_cast<const uint4*>(a.norm_w + q * 8));
    }
    named_bar(kBarConsumers, kConsumers);
  }
}

// stage_x for an input that is a deferred residual sum (persistent step): x = bf16(res + bf16(sum)) with
// res = a.x (the residual stream before the projection) and sum = fx_to_float(fxs) (the projection's
// fixed-point group sums) - the RES epilogue's arithmetic - then RMSNorm-ed as stage_x does. This CTA
// also writes its share of x (chunks q = cta, cta + G, ...) to xw, the residual stream's next buffer.
// 256 threads; kFxStage chunks of 8 values (and their 8 sums) per thread in flight.
template <int M>
__device__ void stage_x_fx(const GemvArgs& a, const int64_t* fxs, __nv_bfloat16* xw, int cta, int G,
                           __nv_bfloat16* xs, float* wsum, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int kv8 = (int)(a.k >> 3);
  for (int m = 0; m < M; ++m) {
    float sq = 0.f;
    for (int q0 = 0; q0 < kv8; q0 += kFxStage * kConsumers) {
      uint4 rv[kFxStage];
      longlong2 sv[kFxStage][4];
#pragma unroll
      for (int j = 0; j < kFxStage; ++j) {
        const int q = q0 + j * kConsumers + tid;
        if (q < kv8) {
          rv[j] = ld_cg_v4(a.x + m * a.ldx + q * 8);
          const longlong2* sp = reinterpret_cast<const longlong2*>(fxs + (int64_t)m * a.k + q * 8);
#pragma unroll
          for (int e = 0; e < 4; ++e) sv[j][e] = __ldcg(sp + e);
        }
      }
#pragma unroll
      for (int j = 0; j < kFxStage; ++j) {
        const int q = q0 + j * kConsumers + tid;
        if (q >= kv8) continue;
        const uint32_t ru[4] = {rv[j].x, rv[j].y, rv[j].z, rv[j].w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float lo = bf16r(bf_lo(ru[e]) + bf16r(fx_to_float(sv[j][e].x)));
          const float hi = bf16r(bf_hi(ru[e]) + bf16r(fx_to_float(sv[j][e].y)));
          o[e] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
          if (a.norm_w) {
            sq = fmaf(lo, lo, sq);
            sq = fmaf(hi, hi, sq);
          }
        }
        const uint4 v = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(xs + (int64_t)m * a.k + q * 8) = v;
        if (xw && q % G == cta) *reinterpret_cast<uint4*>(xw + m * a.ldx + q * 8) = v;
      }
    }
    if (a.norm_w) {
      sq = warp_sum(sq);
      if (lane == 0) wsum[m * kConsumerWarps + warp] = sq;
    }
  }
  named_bar(kBarConsumers, kConsumers);
  if (a.norm_w) {
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
    named_bar(kBarConsumers, kConsumers);
  }
}

// ------------------------------------------------------------------ epilogues (256 consumer threads)
template <int M>
constexpr int res_per() {  // residual values per thread
  return (M * kBlockRows + kConsumers - 1) / kConsumers;
}

// Residual values of group g this thread's epilogue adds (one L2 round trip for all of them).
template <int M>
__device__ __forceinline__ void load_res(const GemvArgs& a, int g, int tid, float* rv) {
  constexpr int kResPer = res_per<M>();
#pragma unroll
  for (int j = 0; j < kResPer; ++j) {
    const int idx = tid + j * kConsumers;
    if (idx < a.m_act * kBlockRows) {
      const int m = idx >> 7, r = idx & 127;
      const uint16_t rb = __ldcg(reinterpret_cast<const unsigned short*>(a.res + m * a.ldr + (int64_t)g * kBlockRows + r));
      rv[j] = __uint_as_float((uint32_t)rb << 16);
    }
  }
}

template <int M, int MODE>
__device__ void finalize_group(const GemvArgs& a, int g, float* red, float* wsum, float* lmv, int* lmi,
                               const float* aux, const int* flags, int tid, const float* res_pre = nullptr) {
  const int MA = a.m_act;  // rows to emit (the rest of the M are padding)
  if constexpr (MODE == MODE_STORE || MODE == MODE_RES) {
    constexpr int kResPer = res_per<M>();
    float rv[kResPer];
    if constexpr (MODE == MODE_RES) {
      if (res_pre) {
#pragma unroll
        for (int j = 0; j < kResPer; ++j) rv[j] = res_pre[j];
      } else {
        load_res<M>(a, g, tid, rv);
      }
    }
#pragma unroll
    for (int j = 0; j < kResPer; ++j) {
      const int idx = tid + j * kConsumers;
      if (idx >= MA * kBlockRows) continue;
      const int m = idx >> 7, r = idx & 127;
      const int64_t n = (int64_t)g * kBlockRows + r;
      float v = bf16r(red[idx]);
      if constexpr (MODE == MODE_RES) v = rv[j] + v;
      a.out[m * a.ldo + n] = __float2bfloat16_rn(v);
    }
  } else if constexpr (MODE == MODE_SWIGLU) {
    for (int idx = tid; idx < MA * 64; idx += kConsumers) {
      const int m = idx >> 6, j = idx & 63;
      const float gv = bf16r(red[m * kBlockRows + j]);
      const float uv = bf16r(red[m * kBlockRows + 64 + j]);
      const float s = bf16r(gv / (1.0f + expf(-gv)));
      if (a.out_npad)  // output column g * 64 + j is column j of K-block g of the next projection
        a.out[((int64_t)g * a.out_npad + m) * 64 + (((j >> 3) ^ (m & 7)) << 3) + (j & 7)] =
            __float2bfloat16_rn(s * uv);
      else
        a.out[m * a.ldo + (int64_t)g * 64 + j] = __float2bfloat16_rn(s * uv);
    }
  } else if constexpr (MODE == MODE_QKV) {
    const int64_t p = flags[2];  // position and its RoPE row were loaded once per op (aux)
    const int lane = tid & 31;
    if (p < 0) return;           // out-of-range position: flagged, nothing written
    // BF16 projection output
    for (int idx = tid; idx < MA * kBlockRows; idx += kConsumers) {
      const float v = bf16r(red[idx]);
      red[idx] = v;
      if (a.raw_out) a.raw_out[(idx >> 7) * a.n + (int64_t)g * kBlockRows + (idx & 127)] = __float2bfloat16_rn(v);
    }
    if (g >= a.nq + a.nkv) {  // V head: append as is
      const int kvh = g - a.nq - a.nkv;
      for (int idx = tid; idx < MA * kBlockRows; idx += kConsumers) {
        const int m = idx >> 7, r = idx & 127;
        a.v_cache[m * a.cs_b + kvh * a.cs_h + p * 128 + r] = __float2bfloat16_rn(red[idx]);
      }
      return;
    }
    // per-head RMSNorm (Qwen3RMSNorm over 128): sum of squares per activation row
    for (int base = 0; base < MA * kBlockRows; base += kConsumers) {
      const int idx = base + tid;
      float sq = 0.f;
      if (idx < MA * kBlockRows) sq = red[idx] * red[idx];
      sq = warp_sum(sq);
      if (lane == 0 && idx < MA * kBlockRows) wsum[idx >> 5] = sq;  // one slot per 32 rows
    }
    named_bar(kBarConsumers, kConsumers);
    const float* nw = aux + (g < a.nq ? 256 : 384);  // q_norm / k_norm, loaded once per op
    for (int idx = tid; idx < MA * kBlockRows; idx += kConsumers) {
      const int m = idx >> 7, r = idx & 127;
      const float var = (wsum[m * 4 + 0] + wsum[m * 4 + 1] + wsum[m * 4 + 2] + wsum[m * 4 + 3]) / 128.0f;
      const float rstd = 1.0f / sqrtf(var + a.eps);
      const float y = bf16r(nw[r] * bf16r(red[idx] * rstd));
      red[idx] = y;  // each thread rewrites only its own entries; partners are read after the barrier
    }
    named_bar(kBarConsumers, kConsumers);
    for (int idx = tid; idx < MA * kBlockRows; idx += kConsumers) {
      const int m = idx >> 7, r = idx & 127;
      const float y = red[idx];
      const float yp = red[(idx & ~127) | (r ^ 64)];
      const float c = aux[r];
      const float s = aux[128 + r];
      // q*cos + rotate_half(q)*sin with every product a BF16 tensor (rotate_half = cat(-q2, q1))
      const float rot = (r < 64) ? bf16r(-yp * s) : bf16r(yp * s);
      const __nv_bfloat16 o = __float2bfloat16_rn(bf16r(y * c) + rot);
      if (g < a.nq) {
        a.q_out[((int64_t)m * a.nq + g) * 128 + r] = o;
      } else {
        a.k_cache[m * a.cs_b + (g - a.nq) * a.cs_h + p * 128 + r] = o;
      }
    }
  } else if constexpr (MODE == MODE_LM) {
    const int lane = tid & 31;
    for (int base = 0; base < MA * kBlockRows; base += kConsumers) {
      const int idx = base + tid;
      float v = -INFINITY;
      int n = 0x7fffffff;
      if (idx < MA * kBlockRows) {
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
      if (lane == 0 && idx < MA * kBlockRows) {
        wsum[(idx >> 5) * 2] = v;
        reinterpret_cast<int*>(wsum)[(idx >> 5) * 2 + 1] = n;
      }
    }
    named_bar(kBarConsumers, kConsumers);
    if (tid < MA) {
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
  }
}

// Optional timeline hook of the segment flush (a kernel that defines it before including this header
// records its phases); a no-op otherwise.
#ifndef QD_FLUSH_HOOK
#define QD_FLUSH_HOOK(k, flags, tid) \
  do {                                \
  } while (0)
#endif

// A CTA's segment of row group g (blocks seg_first..b) is reduced into red[m * 128 + r]. If the segment is
// the whole group, run the epilogue; otherwise store the partial, take the group's ticket, and the CTA
// that completes the group sums all partials in CTA order and runs the epilogue. 256 consumer threads.
// FXSUM: the fixed-point group sums are compiled in (the CUDA-core kernels, M <= 8 activation rows; the
// tensor-core kernels, whose N is 16..64, never use them and so carry none of their registers).
template <int M, int MODE, bool DEFER = false, bool FXSUM = (M <= 8)>
__device__ void flush_segment(const GemvArgs& a, int g, int64_t seg_first, int64_t b, int cta, float* red,
                              float* wsum, float* lmv, int* lmi, float* aux, int* flags, int tid) {
  const int64_t gb0 = (int64_t)g * a.kblocks;
  const int nseg_blk = (int)(b + 1 - seg_first);
  bool finalized = false;
  if constexpr (DEFER) {  // every segment into the fixed-point sums (a.fx), no epilogue here
    for (int idx = tid; idx < a.m_act * kBlockRows; idx += kConsumers) {
      unsigned long long* dst = reinterpret_cast<unsigned long long*>(a.fx + (int64_t)(idx >> 7) * a.n +
                                                                      (int64_t)g * kBlockRows + (idx & 127));
      atomicAdd(dst, (unsigned long long)fx_of(red[idx]));
    }
    named_bar(kBarConsumers, kConsumers);
    if (tid == 0 && a.fx_ctr) red_release_add(a.fx_ctr, nseg_blk);  // releases this CTA's additions
    named_bar(kBarConsumers, kConsumers);
    return;
  }
  if (FXSUM && (MODE == MODE_RES || MODE == MODE_QKV) && a.fx_numerics && seg_first == gb0 &&
      nseg_blk == a.kblocks) {
    // the whole group in this CTA: the value a fixed-point sum of one contribution gives
    for (int idx = tid; idx < a.m_act * kBlockRows; idx += kConsumers) red[idx] = fx_to_float(fx_of(red[idx]));
    named_bar(kBarConsumers, kConsumers);
    finalize_group<M, MODE>(a, g, red, wsum, lmv, lmi, aux, flags, tid);
    finalized = true;
  } else if (seg_first == gb0 && nseg_blk == a.kblocks) {
    finalize_group<M, MODE>(a, g, red, wsum, lmv, lmi, aux, flags, tid);
    finalized = true;
  } else {
    const int c_lo = part_owner(a.total, a.grid, gb0);
    // partials move as float4: kPer per thread, kSB segments' worth of loads in flight at a time
    constexpr int kVec = M * kBlockRows / 4;
    constexpr int kPer = (kVec + kConsumers - 1) / kConsumers;
    constexpr int kSB = kPer >= 4 ? 2 : 8 / kPer;
    float4* dst = reinterpret_cast<float4*>(a.partials + ((int64_t)g * a.smax + (cta - c_lo)) * (M * kBlockRows));
    float4* red4 = reinterpret_cast<float4*>(red);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int q = tid + j * kConsumers;
      if (q < kVec) __stcg(dst + q, red4[q]);
    }
    named_bar(kBarConsumers, kConsumers);
    if (tid == 0) {  // release our partial, acquire the others' when we complete the group
      const int old = atom_add_acq_rel(a.tickets + g, nseg_blk);
      flags[1] = (old + nseg_blk == a.kblocks) ? 1 : 0;
    }
    named_bar(kBarConsumers, kConsumers);
    QD_FLUSH_HOOK(2, flags, tid);
    if (flags[1]) {
      // every CTA in [c_lo, c_hi] owns a non-empty part of the group (T >= G): sum their partials
      // in CTA order
      const int nseg = part_owner(a.total, a.grid, gb0 + a.kblocks - 1) - c_lo + 1;
      const float4* pbase = reinterpret_cast<const float4*>(a.partials + (int64_t)g * a.smax * (M * kBlockRows));
      float res_pre[res_per<M>()];
      if constexpr (MODE == MODE_RES) load_res<M>(a, g, tid, res_pre);  // in flight with the partials
      float4 acc[kPer];
      bool fx_done = false;
      if constexpr (FXSUM && (MODE == MODE_RES || MODE == MODE_QKV)) {
       if (a.fx_numerics) {  // fixed-point group sums (fx_numerics)
        fx_done = true;
        long long iacc[kPer][4];
#pragma unroll
        for (int j = 0; j < kPer; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) iacc[j][e] = 0;
        for (int s0 = 0; s0 < nseg; s0 += kSB) {
          float4 v[kSB][kPer];
#pragma unroll
          for (int b2 = 0; b2 < kSB; ++b2)
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
              const int q = tid + j * kConsumers;
              v[b2][j] = (s0 + b2 < nseg && q < kVec) ? __ldcg(pbase + (int64_t)(s0 + b2) * kVec + q)
                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
          for (int b2 = 0; b2 < kSB; ++b2)
#pragma unroll
            for (int j = 0; j < kPer; ++j)
              if (s0 + b2 < nseg) {
                iacc[j][0] += fx_of(v[b2][j].x);
                iacc[j][1] += fx_of(v[b2][j].y);
                iacc[j][2] += fx_of(v[b2][j].z);
                iacc[j][3] += fx_of(v[b2][j].w);
              }
        }
#pragma unroll
        for (int j = 0; j < kPer; ++j)
          acc[j] = make_float4(fx_to_float(iacc[j][0]), fx_to_float(iacc[j][1]), fx_to_float(iacc[j][2]),
                               fx_to_float(iacc[j][3]));
       }
      }
      if (!fx_done) {
#pragma unroll
        for (int j = 0; j < kPer; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < nseg; s0 += kSB) {
          float4 v[kSB][kPer];
#pragma unroll
          for (int b2 = 0; b2 < kSB; ++b2)
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
              const int q = tid + j * kConsumers;
              v[b2][j] = (s0 + b2 < nseg && q < kVec) ? __ldcg(pbase + (int64_t)(s0 + b2) * kVec + q)
                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
          for (int b2 = 0; b2 < kSB; ++b2)
#pragma unroll
            for (int j = 0; j < kPer; ++j)
              if (s0 + b2 < nseg) {
                acc[j].x += v[b2][j].x;
                acc[j].y += v[b2][j].y;
                acc[j].z += v[b2][j].z;
                acc[j].w += v[b2][j].w;
              }
        }
      }
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int q = tid + j * kConsumers;
        if (q < kVec) red4[q] = acc[j];
      }
      named_bar(kBarConsumers, kConsumers);
      QD_FLUSH_HOOK(3, flags, tid);
      finalize_group<M, MODE>(a, g, red, wsum, lmv, lmi, aux, flags, tid, MODE == MODE_RES ? res_pre : nullptr);
      QD_FLUSH_HOOK(4, flags, tid);
      if (tid == 0) atomicExch(a.tickets + g, 0);
      finalized = true;
    }
  }
  if (finalized && a.done) signal_done(a.done, tid);
  named_bar(kBarConsumers, kConsumers);
}

// QKV epilogue inputs, loaded once per op into shared memory: q_norm / k_norm (aux[256..511]) and,
// unless the caller preloaded them (pos_ready), the decode position (flags[2]) and its cos/sin rows
// (aux[0..255]). 256 consumer threads; ends with a barrier.
__device__ __forceinline__ void qkv_prologue(const GemvArgs& a, float* aux, int* flags, int tid) {
  if (tid < 256) aux[256 + tid] = bf16_to_f(tid < 128 ? a.q_norm[tid] : a.k_norm[tid - 128]);
  if (!a.pos_ready) {
    const int64_t p = ld_cg_s64(a.pos);
    const bool in = p >= 0 && p < a.cap;
    if (tid < 128 && in) {
      aux[tid] = bf16_to_f(a.cos[p * 128 + tid]);
      aux[128 + tid] = bf16_to_f(a.sin[p * 128 + tid]);
    }
    if (tid == 0) {
      flags[2] = in ? (int)p : -1;
      if (!in && a.err) atomicOr(a.err, QD_DEVERR_POS);
    }
  }
  named_bar(kBarConsumers, kConsumers);
}

// Consume this CTA's blocks of one projection from the ring (in issue order), flushing a segment
// at every row-group end; ring position (slot, phase) carries across projections.
template <int M, int MODE, bool DEFER = false>
__device__ void consume_blocks(const GemvArgs& a, const Ring& R, int& slot, int& phase, int cta,
                               const __nv_bfloat16* xs, float* red, float* wsum, float* lmv, int* lmi, int* flags,
                               float* aux, int tid, bool& ok) {
  const int warp = tid >> 5, lane = tid & 31;
  if constexpr (MODE == MODE_QKV) qkv_prologue(a, aux, flags, tid);
  const int64_t b_begin = part_begin(a.total, a.grid, cta);
  const int64_t b_end = part_begin(a.total, a.grid, cta + 1);
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

  int64_t seg_first = b_begin;
  int g = (int)(b_begin / a.kblocks);
  int kb = (int)(b_begin - (int64_t)g * a.kblocks) - 1;
  for (int64_t b = b_begin; b < b_end; ++b) {
    if (++kb == a.kblocks) {
      kb = 0;
      ++g;
    }
    if (ok) ok = mbar_wait(R.full(slot), phase, a.err, kErrWaitFull);
    {
      const char* blk = R.base + slot * kBlockBytes;
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
    if (lane == 0) mbar_arrive(R.empty(slot));
    if (++slot == R.nst) {
      slot = 0;
      phase ^= 1;
    }

    const bool seg_end = (kb == a.kblocks - 1) || (b == b_end - 1);
    if (!seg_end) continue;

    // ------------------------------------------------------------ flush the segment of group g
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
    named_bar(kBarConsumers, kConsumers);
    flush_segment<M, MODE, DEFER>(a, g, seg_first, b, cta, red, wsum, lmv, lmi, aux, flags, tid);
    seg_first = b + 1;
  }
}

// Global argmax over the CTAs' per-row bests (LM head): each CTA posts its best, the last CTA to arrive
// reduces all of them (lowest index on exact ties) and writes tok. Returns true in that last CTA.
template <int M>
__device__ bool lm_global_argmax(const GemvArgs& a, int cta, float* wsum, float* lmv, int* lmi, int* flags, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  if (tid < a.m_act) {
    a.cta_val[tid * a.grid + cta] = lmv[tid];
    a.cta_idx[tid * a.grid + cta] = lmi[tid];
  }
  named_bar(kBarConsumers, kConsumers);
  if (tid == 0) flags[1] = (atom_add_acq_rel(a.lm_ticket, 1) == a.grid - 1) ? 1 : 0;
  named_bar(kBarConsumers, kConsumers);
  if (!flags[1]) return false;
  // one warp per activation row: lanes stride over the CTAs' candidates, then a shuffle reduction
  for (int m = warp; m < a.m_act; m += kConsumerWarps) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll 4
    for (int q = lane; q < a.grid; q += 32) {
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
    if (lane == 0) a.tok[m] = (int64_t)bi;
  }
  if (tid == 0) {
    if (a.inc_pos && a.pos_inc) a.pos_inc[0] = ld_cg_s64(a.pos_inc) + 1;
    atomicExch(a.lm_ticket, 0);
  }
  return true;
}

}  // namespace qd
