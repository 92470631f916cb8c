// Device side of the split-K GQA flash-decode, shared by the attention kernel (qd_attn.cu) and the
// persistent decode-step kernel (qd_step.cu).
//
// A unit is (sequence b, KV head, split): a team of 4 warps serves the GROUP = 4 query heads of that
// KV head over one contiguous key range of the static cache, so each K/V row is read from HBM once
// per step. The valid length (pos + 1) is read on the device; keys at or beyond it are never read.
//
// Each warp takes 8 keys per pass (the team covers 32 consecutive keys), all of the pass's loads
// issued before any is used, so a pass costs one memory latency. For q.k four lanes share a key, each
// summing 32 of the 128 dims (fp32 FMAs of BF16 inputs) before two shuffles combine them; the warp
// keeps a running max / sum with fp32 probabilities, rounds them to BF16 and accumulates P.V with
// lane j holding dims 4j..4j+3 - the flash-attention arithmetic of the reference's SDPA and Triton
// kernels (engine/kernels/decode_attn.py:1-11). The four warps'
// states merge in shared memory; the unit writes (acc, max, sum) for its split, and the last split to
// arrive (atomic ticket) merges all splits in split order (engine/kernels/decode_attn.py:73-86):
//   w_s = exp(m_s - max_s m_s), out = sum_s acc_s w_s / sum_s l_s w_s.
#pragma once

#include "qd_common.cuh"
#include "qd_host.h"

namespace qd {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kGroup = 4;  // query heads per KV head (Qwen3-4B: 32 / 8)
constexpr int kHeadDim = 128;

struct AttnArgs {
  const __nv_bfloat16 *q, *k, *v;
  const int64_t* pos;
  __nv_bfloat16* out;
  int batch, nq, nkv, splits;
  int64_t cap, cs_b, cs_h, chunk;
  float scale;
  float* part_acc;
  float* part_ml;
  int* tickets;
  int* err;
  int* done;  // optional: +1 (release) per merged (sequence, KV head), or per unit with partials_only
  int keys_per_split;  // splits in use at a given length: ~this many keys each, at most `splits`
  int partials_only;   // every unit leaves its (acc, max, sum) and signals; the reader merges them
};

// Valid length (pos + 1) clamped to the cache; flags QD_DEVERR_POS when the position is outside it.
__device__ __forceinline__ int64_t attn_len_at(int64_t pos, int64_t cap, int* err, bool flag) {
  int64_t len = pos + 1;
  if (len < 1 || len > cap) {
    if (flag && err) atomicOr(err, QD_DEVERR_POS);
    len = len < 1 ? 1 : cap;
  }
  return len;
}
__device__ __forceinline__ int64_t attn_len(const AttnArgs& a, int64_t pos, bool flag) {
  return attn_len_at(pos, a.cap, a.err, flag);
}

// Splits in use at length len (every unit computes the same value): about keys_per_split keys each,
// at most a.splits, chunk a multiple of 32 keys (one pass of the 4 warps).
__device__ __forceinline__ int attn_active(const AttnArgs& a, int64_t len, int64_t* chunk) {
  const int64_t kps = a.keys_per_split > 0 ? a.keys_per_split : a.chunk;
  int64_t n = (len + kps - 1) / kps;
  if (n > a.splits) n = a.splits;
  if (n < 1) n = 1;
  int64_t c = (len + n - 1) / n;
  c = (c + 31) / 32 * 32;
  *chunk = c;
  return (int)((len + c - 1) / c);
}

// 16-byte aligned and sized (the q.k loop reads qs as float4; the step kernel places two of these
// back to back).
struct __align__(16) AttnSmem {
  float qs[kGroup][kHeadDim];
  float wacc[kAttnWarps][kGroup][kHeadDim];
  float wm[kAttnWarps][kGroup], wl[kAttnWarps][kGroup];
  int last_flag;
};

// One unit on a team of 128 threads (team thread id `tid`, named barrier `bar_id`); `len` is the valid
// length (attn_len). Units past the splits in use at this length return at once.
// q_ready: the caller has already put the unit's 4 query heads (BF16 values as floats) into sm.qs.
static __device__ void attn_unit(const AttnArgs& a, int b, int kvh, int split, int tid, int bar_id, AttnSmem& sm,
                                 int64_t len, bool q_ready = false) {
  const int warp = tid >> 5, lane = tid & 31;
  int64_t chunk;
  const int n_use = attn_active(a, len, &chunk);
  if (split >= n_use) return;
  const int64_t start = (int64_t)split * chunk;
  int64_t end = start + chunk;
  if (end > len) end = len;

  if (!q_ready) {
    for (int h = 0; h < kGroup; ++h) {
      const __nv_bfloat16* qp = a.q + ((int64_t)b * a.nq + kvh * kGroup + h) * kHeadDim;
      const uint16_t u = __ldcg(reinterpret_cast<const unsigned short*>(qp) + tid);
      sm.qs[h][tid] = __uint_as_float((uint32_t)u << 16);
    }
  }
  named_bar(bar_id, kAttnThreads);

  const __nv_bfloat16* kbase = a.k + (int64_t)b * a.cs_b + (int64_t)kvh * a.cs_h;
  const __nv_bfloat16* vbase = a.v + (int64_t)b * a.cs_b + (int64_t)kvh * a.cs_h;
  float m_run[kGroup], l_run[kGroup], acc[kGroup][4];
#pragma unroll
  for (int h = 0; h < kGroup; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.f;
#pragma unroll
    for (int d = 0; d < 4; ++d) acc[h][d] = 0.f;
  }

  // Each warp takes 8 keys per pass (the 4 warps cover 32 consecutive keys): for q.k, lane = (key
  // lane / 4, quarter lane % 4 of the 128 dims); for P.V, lane = dims 4 lane .. 4 lane + 3.
  const int kj = lane >> 2, qd = lane & 3;
  for (int64_t t0 = start + warp * 8; t0 < end; t0 += kAttnWarps * 8) {
    const int64_t key = t0 + kj;
    const bool valid = key < end;
    const int nk = (int)((end - t0) < 8 ? (end - t0) : 8);
    // all of the pass's loads in flight first
    uint4 kr[4];
    const __nv_bfloat16* kp = kbase + (valid ? key : t0) * kHeadDim + qd * 32;
#pragma unroll
    for (int c = 0; c < 4; ++c) kr[c] = ld_cg_v4(kp + c * 8);
    uint2 vr[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) vr[j] = (j < nk) ? ld_cg_v2(vbase + (t0 + j) * kHeadDim + 4 * lane) : make_uint2(0u, 0u);
    float s[kGroup] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float kf[8] = {bf_lo(kr[c].x), bf_hi(kr[c].x), bf_lo(kr[c].y), bf_hi(kr[c].y),
                           bf_lo(kr[c].z), bf_hi(kr[c].z), bf_lo(kr[c].w), bf_hi(kr[c].w)};
#pragma unroll
      for (int h = 0; h < kGroup; ++h) {
        const float4 q0 = *reinterpret_cast<const float4*>(&sm.qs[h][qd * 32 + c * 8]);
        const float4 q1 = *reinterpret_cast<const float4*>(&sm.qs[h][qd * 32 + c * 8 + 4]);
        s[h] = fmaf(q0.x, kf[0], s[h]);
        s[h] = fmaf(q0.y, kf[1], s[h]);
        s[h] = fmaf(q0.z, kf[2], s[h]);
        s[h] = fmaf(q0.w, kf[3], s[h]);
        s[h] = fmaf(q1.x, kf[4], s[h]);
        s[h] = fmaf(q1.y, kf[5], s[h]);
        s[h] = fmaf(q1.z, kf[6], s[h]);
        s[h] = fmaf(q1.w, kf[7], s[h]);
      }
    }
    float pb[kGroup];
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      s[h] += __shfl_xor_sync(0xffffffffu, s[h], 1);  // the 4 quarters of key kj
      s[h] += __shfl_xor_sync(0xffffffffu, s[h], 2);
      const float sc = valid ? s[h] * a.scale : -INFINITY;
      // the 4 lanes of a key now agree: reduce over the 8 keys (lane bits 2..4) only
      float mt = sc;
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
      const float m_new = fmaxf(m_run[h], mt);
      const float alpha = expf(m_run[h] - m_new);  // exp(-inf) = 0 on the first pass
      const float p = valid ? expf(sc - m_new) : 0.f;
      float ps = p;  // each key counted once
      ps += __shfl_xor_sync(0xffffffffu, ps, 4);
      ps += __shfl_xor_sync(0xffffffffu, ps, 8);
      ps += __shfl_xor_sync(0xffffffffu, ps, 16);
      l_run[h] = l_run[h] * alpha + ps;
#pragma unroll
      for (int d = 0; d < 4; ++d) acc[h][d] *= alpha;
      m_run[h] = m_new;
      pb[h] = bf16r(p);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float vf[4] = {bf_lo(vr[j].x), bf_hi(vr[j].x), bf_lo(vr[j].y), bf_hi(vr[j].y)};
#pragma unroll
      for (int h = 0; h < kGroup; ++h) {
        const float pj = __shfl_sync(0xffffffffu, pb[h], j * 4);  // 0 for keys past the end
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[h][d] = fmaf(pj, vf[d], acc[h][d]);
      }
    }
  }

  // merge the four warps of this unit
#pragma unroll
  for (int h = 0; h < kGroup; ++h) {
#pragma unroll
    for (int d = 0; d < 4; ++d) sm.wacc[warp][h][4 * lane + d] = acc[h][d];
    if (lane == 0) {
      sm.wm[warp][h] = m_run[h];
      sm.wl[warp][h] = l_run[h];
    }
  }
  named_bar(bar_id, kAttnThreads);
  const int64_t row0 = ((int64_t)b * a.nq + kvh * kGroup) * a.splits;
  if (!a.partials_only && n_use == 1) {  // one split covers every key: normalise and write, no merge
    for (int h = 0; h < kGroup; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, sm.wm[w][h]);
      float num = 0.f, den = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        if (sm.wm[w][h] == -INFINITY) continue;
        const float sc = expf(sm.wm[w][h] - mx);
        num = fmaf(sm.wacc[w][h][tid], sc, num);
        den = fmaf(sm.wl[w][h], sc, den);
      }
      // as the merge of one split computes it: weight exp(0) = 1
      a.out[((int64_t)b * a.nq + kvh * kGroup + h) * kHeadDim + tid] =
          __float2bfloat16_rn(fmaf(num, 1.0f, 0.f) / fmaf(den, 1.0f, 0.f));
    }
    if (a.done) {
      named_bar(bar_id, kAttnThreads);
      if (tid == 0) red_release_add(a.done, 1);
    }
    named_bar(bar_id, kAttnThreads);
    return;
  }
  for (int h = 0; h < kGroup; ++h) {
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, sm.wm[w][h]);
    float num = 0.f, den = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        if (sm.wm[w][h] == -INFINITY) continue;
        const float sc = expf(sm.wm[w][h] - mx);
        num = fmaf(sm.wacc[w][h][tid], sc, num);
        den = fmaf(sm.wl[w][h], sc, den);
      }
    }
    const int64_t part = row0 + (int64_t)h * a.splits + split;
    a.part_acc[part * kHeadDim + tid] = num;
    if (tid == 0) {
      a.part_ml[part * 2] = mx;
      a.part_ml[part * 2 + 1] = den;
    }
  }
  named_bar(bar_id, kAttnThreads);
  if (a.partials_only) {  // the consumer merges (attn_merge_partials); release this unit's partial
    if (tid == 0 && a.done) red_release_add(a.done, 1);
    named_bar(bar_id, kAttnThreads);
    return;
  }
  if (tid == 0)
    sm.last_flag = (atom_add_acq_rel(a.tickets + (int64_t)b * a.nkv + kvh, 1) == n_use - 1) ? 1 : 0;
  named_bar(bar_id, kAttnThreads);
  if (sm.last_flag) {
    // Merge the splits that hold keys (those past the valid length have max -inf and weight 0), in
    // split order. (max, sum) of every head and split go through shared memory (the warp-merge
    // buffer is free by now), then each thread combines its dimension for the 4 heads with all of
    // its accumulator loads in flight.
    const int n_act = n_use;  // every split in use holds at least one key
    float* mm = &sm.wacc[0][0][0];  // [kGroup][n_act] maxima, then sums, then weights
    float* ll = mm + kGroup * n_act;
    float* ww = ll + kGroup * n_act;
    for (int t = tid; t < kGroup * n_act; t += kAttnThreads) {
      const int h = t / n_act, sp = t - h * n_act;
      const int64_t part = row0 + (int64_t)h * a.splits + sp;
      mm[t] = ld_cg_f32(a.part_ml + part * 2);
      ll[t] = ld_cg_f32(a.part_ml + part * 2 + 1);
    }
    named_bar(bar_id, kAttnThreads);
    for (int t = tid; t < kGroup * n_act; t += kAttnThreads) {
      const int h = t / n_act;
      float mx = -INFINITY;
      for (int sp = 0; sp < n_act; ++sp) mx = fmaxf(mx, mm[h * n_act + sp]);
      ww[t] = (mm[t] == -INFINITY) ? 0.f : expf(mm[t] - mx);
    }
    named_bar(bar_id, kAttnThreads);
    float num[kGroup] = {0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < n_act; s0 += 8) {
      float av[kGroup][8];
#pragma unroll
      for (int h = 0; h < kGroup; ++h)
#pragma unroll
        for (int j = 0; j < 8; ++j)
          av[h][j] = (s0 + j < n_act)
                         ? ld_cg_f32(a.part_acc + (row0 + (int64_t)h * a.splits + s0 + j) * kHeadDim + tid)
                         : 0.f;
#pragma unroll
      for (int h = 0; h < kGroup; ++h)
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (s0 + j < n_act) num[h] = fmaf(av[h][j], ww[h * n_act + s0 + j], num[h]);
    }
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      float den = 0.f;
      for (int sp = 0; sp < n_act; ++sp) den = fmaf(ll[h * n_act + sp], ww[h * n_act + sp], den);
      a.out[((int64_t)b * a.nq + kvh * kGroup + h) * kHeadDim + tid] = __float2bfloat16_rn(num[h] / den);
    }
    if (tid == 0) atomicExch(a.tickets + (int64_t)b * a.nkv + kvh, 0);
    if (a.done) {
      named_bar(bar_id, kAttnThreads);
      if (tid == 0) red_release_add(a.done, 1);
    }
  }
  named_bar(bar_id, kAttnThreads);  // shared memory is reused by the team's next unit
}

}  // namespace qd
