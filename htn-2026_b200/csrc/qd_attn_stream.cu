// Streaming split-K GQA flash-decode for large batch x length, sm_100a.
//
// The work is the key range of every (sequence, KV head) pair in 32-key chunks, T = pairs x chunks,
// dealt out stream-K style: CTA c of G takes chunks [c T / G, (c + 1) T / G), which may end one pair
// and start the next, so every CTA streams the same number of bytes whatever the batch and length.
// A producer warp moves each chunk's K and V rows (contiguous in the [B, nkv, cap, 128] cache) into a
// shared-memory ring with 1-D bulk copies; eight consumer warps compute, for the GROUP = 4 query heads
// of the pair, q.k (each lane 4 dims, a fixed-order butterfly across the warp), the online softmax
// (one warp per head: running max and sum in fp32, probabilities rounded to BF16 for P.V as the
// reference's SDPA / Triton kernels do, engine/kernels/decode_attn.py:1-11) and P.V (each thread 2
// dims x 8 keys of the chunk). A CTA that covers a whole pair writes the output; otherwise it writes
// (acc, max, sum) for its segment, and the last segment to arrive (atomic ticket counting chunks)
// merges the pair's segments in CTA order (engine/kernels/decode_attn.py:73-86):
//   w_s = exp(m_s - max_s m_s), out = sum_s acc_s w_s / sum_s l_s w_s.
#include "qd_attn_dev.cuh"
#include "qd_plan.h"

namespace qd {

constexpr int kSChunk = 32;                              // keys per chunk (one ring stage)
constexpr int kSStageBytes = 2 * kSChunk * kHeadDim * 2;  // K rows then V rows: 16 KiB
constexpr int kSConsumerWarps = 8;
constexpr int kSConsumers = kSConsumerWarps * 32;
constexpr int kSThreads = kSConsumers + 32;
constexpr int kSBar = 1;  // named barrier of the 256 consumer threads
constexpr int kSStages = 4;
constexpr int kSCtasPerSm = 3;

struct StreamArgs {
  const __nv_bfloat16 *q, *k, *v;
  const int64_t* pos;
  __nv_bfloat16* out;
  int batch, nq, nkv, grid, smax;
  int64_t cap, cs_b, cs_h;
  float scale;
  float* part_acc;  // [pairs][smax][4][128]
  float* part_ml;   // [pairs][smax][4][2]
  int* tickets;     // [pairs], chunks arrived
  int* err;
};

struct __align__(16) StreamSmem {
  char ring[kSStages][kSStageBytes];
  float s[kSChunk][kGroup];     // scaled scores of the chunk
  float p[kSChunk][kGroup];     // BF16-rounded probabilities
  float alpha[kGroup];          // rescale of the running accumulators for this chunk
  float ml[kGroup][2];          // running max / sum at a segment end
  float wacc[4][kGroup][kHeadDim];  // the four key quarters' accumulators; merge staging after that
  int flag, issued;
  uint64_t full[kSStages], empty[kSStages];
};

__device__ __forceinline__ void stream_flush(const StreamArgs& a, StreamSmem& sm, int pair, int seg_first,
                                             int seg_last, int nch, int64_t T, int G, int cta,
                                             float (&acc)[kGroup][2], int tid) {
  const int dp = tid & 63, kq = tid >> 6;
  // the four key quarters' accumulators -> per (head, dim) sums, in quarter order
#pragma unroll
  for (int h = 0; h < kGroup; ++h) {
    sm.wacc[kq][h][2 * dp] = acc[h][0];
    sm.wacc[kq][h][2 * dp + 1] = acc[h][1];
  }
  named_bar(kSBar, kSConsumers);
  const int b = pair / a.nkv, kvh = pair - b * a.nkv;
  const int64_t orow = ((int64_t)b * a.nq + kvh * kGroup) * kHeadDim;
  float num[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int idx = tid + j * kSConsumers, h = idx >> 7, d = idx & 127;
    num[j] = ((sm.wacc[0][h][d] + sm.wacc[1][h][d]) + sm.wacc[2][h][d]) + sm.wacc[3][h][d];
  }
  if (seg_first == 0 && seg_last == nch - 1) {  // the whole pair: normalise and write
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int idx = tid + j * kSConsumers, h = idx >> 7, d = idx & 127;
      a.out[orow + h * kHeadDim + d] = __float2bfloat16_rn(num[j] / sm.ml[h][1]);
    }
    named_bar(kSBar, kSConsumers);  // wacc / ml are reused by the next segment
    return;
  }
  const int64_t gc0 = (int64_t)pair * nch;
  const int c_lo = part_owner(T, G, gc0);
  const int slot = cta - c_lo;
  if (slot < 0 || slot >= a.smax) {  // cannot happen with the host plan's smax; never write out of bounds
    if (tid == 0 && a.err) atomicOr(a.err, kErrDep);
    named_bar(kSBar, kSConsumers);
    return;
  }
  const int64_t prow = ((int64_t)pair * a.smax + slot) * kGroup;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int idx = tid + j * kSConsumers, h = idx >> 7, d = idx & 127;
    __stcg(a.part_acc + (prow + h) * kHeadDim + d, num[j]);
  }
  if (tid < 2 * kGroup) __stcg(a.part_ml + prow * 2 + tid, (&sm.ml[0][0])[tid]);
  named_bar(kSBar, kSConsumers);
  if (tid == 0) {
    const int n = seg_last - seg_first + 1;
    sm.flag = (atom_add_acq_rel(a.tickets + pair, n) + n == nch) ? 1 : 0;
  }
  named_bar(kSBar, kSConsumers);
  const int nseg = part_owner(T, G, gc0 + nch - 1) - c_lo + 1;
  if (sm.flag && nseg > a.smax) {  // cannot happen with the host plan's smax; never read out of bounds
    if (tid == 0 && a.err) atomicOr(a.err, kErrDep);
  } else if (sm.flag) {
    float* mm = &sm.wacc[0][0][0];  // [kGroup][nseg] maxima, sums, weights
    float* ll = mm + kGroup * nseg;
    float* ww = ll + kGroup * nseg;
    const int64_t prow0 = (int64_t)pair * a.smax * kGroup;
    for (int t = tid; t < kGroup * nseg; t += kSConsumers) {
      const int h = t / nseg, s = t - h * nseg;
      mm[t] = ld_cg_f32(a.part_ml + (prow0 + (int64_t)s * kGroup + h) * 2);
      ll[t] = ld_cg_f32(a.part_ml + (prow0 + (int64_t)s * kGroup + h) * 2 + 1);
    }
    named_bar(kSBar, kSConsumers);
    for (int t = tid; t < kGroup * nseg; t += kSConsumers) {
      const int h = t / nseg;
      float mx = -INFINITY;
      for (int s = 0; s < nseg; ++s) mx = fmaxf(mx, mm[h * nseg + s]);
      ww[t] = (mm[t] == -INFINITY) ? 0.f : expf(mm[t] - mx);
    }
    named_bar(kSBar, kSConsumers);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int idx = tid + j * kSConsumers, h = idx >> 7, d = idx & 127;
      float nm = 0.f;
      for (int s0 = 0; s0 < nseg; s0 += 8) {
        float av[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          av[i] = (s0 + i < nseg) ? ld_cg_f32(a.part_acc + (prow0 + (int64_t)(s0 + i) * kGroup + h) * kHeadDim + d)
                                  : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (s0 + i < nseg) nm = fmaf(av[i], ww[h * nseg + s0 + i], nm);
      }
      float den = 0.f;
      for (int s = 0; s < nseg; ++s) den = fmaf(ll[h * nseg + s], ww[h * nseg + s], den);
      a.out[orow + h * kHeadDim + d] = __float2bfloat16_rn(nm / den);
    }
    if (tid == 0) atomicExch(a.tickets + pair, 0);
  }
  named_bar(kSBar, kSConsumers);
}

__global__ void __launch_bounds__(kSThreads, kSCtasPerSm) attn_stream_kernel(const __grid_constant__ StreamArgs a) {
  extern __shared__ __align__(16) char smem_raw[];
  StreamSmem& sm = *reinterpret_cast<StreamSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kSStages; ++s) {
      mbar_init(smem_u32(&sm.full[s]), 1);
      mbar_init(smem_u32(&sm.empty[s]), kSConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  grid_dep_wait();  // q and the new token's K/V come from the preceding kernel
  grid_dep_launch();
  const int64_t len = attn_len_at(ld_cg_s64(a.pos), a.cap, a.err, tid == 0 && cta == 0);
  const int nch = (int)((len + kSChunk - 1) / kSChunk);
  const int pairs = a.batch * a.nkv;
  const int64_t T = (int64_t)pairs * nch;
  // at short lengths fewer chunks than CTAs: deal them over the first T CTAs only, so every CTA of a
  // pair's range [c_lo, c_hi] holds a segment (the merge reads exactly those)
  const int G = (int)(T < a.grid ? T : a.grid);
  if (cta >= G) return;  // no bulk copy was issued and no barrier is pending
  const int64_t c_begin = part_begin(T, G, cta), c_end = part_begin(T, G, cta + 1);

  if (warp == kSConsumerWarps) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int pair = (int)(c_begin / nch), ci = (int)(c_begin - (int64_t)pair * nch);
      int slot = 0, round = 0, issued = 0;
      for (int64_t c = c_begin; c < c_end; ++c) {
        if (round > 0 && !mbar_wait(smem_u32(&sm.empty[slot]), (round - 1) & 1, a.err, kErrWaitEmpty)) break;
        const int b = pair / a.nkv, kvh = pair - b * a.nkv;
        const int64_t k0 = (int64_t)ci * kSChunk;
        const int nk = (int)((len - k0) < kSChunk ? (len - k0) : kSChunk);
        const uint32_t bytes = (uint32_t)nk * kHeadDim * 2;
        const int64_t off = (int64_t)b * a.cs_b + (int64_t)kvh * a.cs_h + k0 * kHeadDim;
        const uint32_t full = smem_u32(&sm.full[slot]);
        mbar_arrive_expect_tx(full, 2 * bytes);
        bulk_g2s(smem_u32(sm.ring[slot]), a.k + off, bytes, full, pol);
        bulk_g2s(smem_u32(sm.ring[slot] + kSStageBytes / 2), a.v + off, bytes, full, pol);
        ++issued;
        if (++ci == nch) {
          ci = 0;
          ++pair;
        }
        if (++slot == kSStages) {
          slot = 0;
          ++round;
        }
      }
      sm.issued = issued;
    }
  } else {
    // ---------------------------------------------------------------- consumers (256 threads)
    const int dp = tid & 63, kq = tid >> 6;
    int pair = (int)(c_begin / nch), ci = (int)(c_begin - (int64_t)pair * nch);
    int seg_first = ci;
    float q[kGroup][4], acc[kGroup][2];
    float m_run = -INFINITY, l_run = 0.f;  // warps 0..3: head `warp`
    auto load_q = [&](int pr) {
      const int b = pr / a.nkv, kvh = pr - b * a.nkv;
#pragma unroll
      for (int h = 0; h < kGroup; ++h) {
        const uint2 u = ld_cg_v2(a.q + ((int64_t)b * a.nq + kvh * kGroup + h) * kHeadDim + 4 * lane);
        q[h][0] = bf_lo(u.x);
        q[h][1] = bf_hi(u.x);
        q[h][2] = bf_lo(u.y);
        q[h][3] = bf_hi(u.y);
#pragma unroll
        for (int e = 0; e < 2; ++e) acc[h][e] = 0.f;
      }
      m_run = -INFINITY;
      l_run = 0.f;
    };
    load_q(pair);
    int slot = 0, phase = 0;
    bool ok = true;
    for (int64_t c = c_begin; c < c_end; ++c) {
      const int64_t k0 = (int64_t)ci * kSChunk;
      const int nk = (int)((len - k0) < kSChunk ? (len - k0) : kSChunk);
      if (ok) ok = mbar_wait(smem_u32(&sm.full[slot]), phase, a.err, kErrWaitFull);
      const char* kst = sm.ring[slot];
      const char* vst = kst + kSStageBytes / 2;
      // q.k: warp w scores keys 4w..4w+3, lane l holds dims 4l..4l+3 of each
      {
        float s[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint2 u = *reinterpret_cast<const uint2*>(kst + (4 * warp + j) * (kHeadDim * 2) + lane * 8);
          const float kf[4] = {bf_lo(u.x), bf_hi(u.x), bf_lo(u.y), bf_hi(u.y)};
#pragma unroll
          for (int h = 0; h < kGroup; ++h) {
            float t = kf[0] * q[h][0];
            t = fmaf(kf[1], q[h][1], t);
            t = fmaf(kf[2], q[h][2], t);
            t = fmaf(kf[3], q[h][3], t);
            s[j * 4 + h] = t;
          }
        }
        // butterfly: after it, lane l holds the full sum of value (l >> 1) & 15 = key j * 4 + head h
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const bool up = lane & 16;
          const float send = up ? s[i] : s[i + 8];
          const float keep = up ? s[i + 8] : s[i];
          s[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const bool up = lane & 8;
          const float send = up ? s[i] : s[i + 4];
          const float keep = up ? s[i + 4] : s[i];
          s[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const bool up = lane & 4;
          const float send = up ? s[i] : s[i + 2];
          const float keep = up ? s[i + 2] : s[i];
          s[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        {
          const bool up = lane & 2;
          const float send = up ? s[0] : s[1];
          const float keep = up ? s[1] : s[0];
          s[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
        }
        s[0] += __shfl_xor_sync(0xffffffffu, s[0], 1);
        if ((lane & 1) == 0) {
          const int v = (lane >> 1) & 15, key = 4 * warp + (v >> 2), h = v & 3;
          sm.s[key][h] = key < nk ? s[0] * a.scale : -INFINITY;
        }
      }
      named_bar(kSBar, kSConsumers);
      // online softmax: warp h over the chunk's 32 keys (lane = key)
      if (warp < kGroup) {
        const float sc = sm.s[lane][warp];
        const float m_new = fmaxf(m_run, warp_max(sc));
        const float alpha = expf(m_run - m_new);  // exp(-inf) = 0 on a segment's first chunk
        const float p = sc == -INFINITY ? 0.f : expf(sc - m_new);
        l_run = l_run * alpha + warp_sum(p);
        m_run = m_new;
        sm.p[lane][warp] = bf16r(p);
        if (lane == 0) sm.alpha[warp] = alpha;
      }
      named_bar(kSBar, kSConsumers);
      // P.V: thread (dims 2 dp, 2 dp + 1; keys 8 kq .. 8 kq + 7)
      {
        const float4 al = *reinterpret_cast<const float4*>(sm.alpha);
        const float alv[4] = {al.x, al.y, al.z, al.w};
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
          acc[h][0] *= alv[h];
          acc[h][1] *= alv[h];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int key = 8 * kq + j;
          if (key < nk) {
            const uint32_t u = *reinterpret_cast<const uint32_t*>(vst + key * (kHeadDim * 2) + dp * 4);
            const float4 pv = *reinterpret_cast<const float4*>(sm.p[key]);
            const float v0 = bf_lo(u), v1 = bf_hi(u);
            const float pw[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
            for (int h = 0; h < kGroup; ++h) {
              acc[h][0] = fmaf(pw[h], v0, acc[h][0]);
              acc[h][1] = fmaf(pw[h], v1, acc[h][1]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sm.empty[slot]));  // this warp is done with the stage
      if (++slot == kSStages) {
        slot = 0;
        phase ^= 1;
      }
      const bool pair_end = (ci == nch - 1) || (c == c_end - 1);
      if (pair_end) {
        if (warp < kGroup && lane == 0) {
          sm.ml[warp][0] = m_run;
          sm.ml[warp][1] = l_run;
        }
        named_bar(kSBar, kSConsumers);
        stream_flush(a, sm, pair, seg_first, ci, nch, T, G, cta, acc, tid);
        if (++ci == nch) {
          ci = 0;
          ++pair;
        }
        seg_first = ci;
        if (c + 1 < c_end) load_q(pair);
      } else {
        ++ci;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {  // never leave with a bulk copy still writing shared memory (bounded waits)
    const int issued = sm.issued;
    for (int it = issued > kSStages ? issued - kSStages : 0; it < issued; ++it)
      if (!mbar_wait(smem_u32(&sm.full[it % kSStages]), (it / kSStages) & 1, a.err, kErrDrain)) break;
  }
}

static int stream_grid(int pairs, int64_t cap, int grid_hint, int* smax_out) {
  const int64_t max_chunks = (int64_t)pairs * ((cap + kSChunk - 1) / kSChunk);
  int64_t g = grid_hint > 0 ? grid_hint : (int64_t)kSCtasPerSm * host_sm_count();
  if (g > (int64_t)79 * pairs) g = (int64_t)79 * pairs;  // keeps smax <= 160 (merge staging in 8 KiB)
  if (g > max_chunks) g = max_chunks;
  if (g < 1) g = 1;
  int64_t smax = 2 * ((g + pairs - 1) / pairs) + 2;
  const int64_t per_pair = (cap + kSChunk - 1) / kSChunk;
  if (smax > per_pair) smax = per_pair;
  *smax_out = (int)smax;
  return (int)g;
}

static int64_t stream_scratch(int pairs, int smax, int64_t* off_ml, int64_t* off_t) {
  const int64_t rows = (int64_t)pairs * smax * kGroup;
  const int64_t acc = (rows * kHeadDim * 4 + 255) / 256 * 256, ml = (rows * 2 * 4 + 255) / 256 * 256;
  *off_ml = acc;
  *off_t = acc + ml;
  return acc + ml + ((int64_t)pairs * 4 + 255) / 256 * 256;
}

}  // namespace qd

using namespace qd;

extern "C" int qd_attn_stream_plan(int batch, int nkv_heads, int64_t cap, int grid_hint, int* grid, int* smax,
                                   int64_t* scratch_bytes) {
  if (batch < 1 || nkv_heads < 1 || cap < 1 || (int64_t)batch * nkv_heads > (1 << 24))
    return set_error(QD_ERR_ARG, "attn stream plan: bad sizes");
  int sm_ = 0;
  const int g = stream_grid(batch * nkv_heads, cap, grid_hint, &sm_);
  int64_t om, ot;
  if (grid) *grid = g;
  if (smax) *smax = sm_;
  if (scratch_bytes) *scratch_bytes = stream_scratch(batch * nkv_heads, sm_, &om, &ot);
  return QD_OK;
}

extern "C" int qd_attn_decode_stream(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos,
                                     void* out, int batch, int nq_heads, int nkv_heads, int64_t cap, int64_t cs_b,
                                     int64_t cs_h, int grid, int smax, float scale, void* scratch,
                                     int64_t scratch_bytes, int* err, int pdl, cudaStream_t stream) {
  if (!q || !k_cache || !v_cache || !pos || !out || !scratch) return set_error(QD_ERR_ARG, "null pointer");
  if (nkv_heads < 1 || nq_heads != nkv_heads * kGroup)
    return set_error(QD_ERR_UNSUPPORTED, "attention is built for %d query heads per KV head", kGroup);
  if (batch < 1 || cap < 1 || (int64_t)batch * nkv_heads > (1 << 24)) return set_error(QD_ERR_ARG, "bad sizes");
  int want_smax = 0;
  const int want_grid = stream_grid(batch * nkv_heads, cap, grid, &want_smax);
  if (grid != want_grid || smax != want_smax)
    return set_error(QD_ERR_ARG, "grid/smax do not match qd_attn_stream_plan (%d, %d)", want_grid, want_smax);
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || cs_h < cap * kHeadDim ||
      cs_b < (int64_t)nkv_heads * cs_h || cs_h % 8 || cs_b % 8)
    return set_error(QD_ERR_ARG, "cache strides/alignment");
  int64_t om, ot;
  const int64_t need = stream_scratch(batch * nkv_heads, smax, &om, &ot);
  if (scratch_bytes < need)
    return set_error(QD_ERR_SCRATCH, "scratch %lld B < %lld B", (long long)scratch_bytes, (long long)need);
  StreamArgs a = {};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k_cache);
  a.v = static_cast<const __nv_bfloat16*>(v_cache);
  a.pos = pos;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.batch = batch;
  a.nq = nq_heads;
  a.nkv = nkv_heads;
  a.grid = grid;
  a.smax = smax;
  a.cap = cap;
  a.cs_b = cs_b;
  a.cs_h = cs_h;
  a.scale = scale;
  char* sc = static_cast<char*>(scratch);
  a.part_acc = reinterpret_cast<float*>(sc);
  a.part_ml = reinterpret_cast<float*>(sc + om);
  a.tickets = reinterpret_cast<int*>(sc + ot);
  a.err = err;
  const int smem = (int)sizeof(StreamSmem);
  if (int rc = set_max_dynamic_smem((const void*)attn_stream_kernel, smem)) return rc;
  return launch_kernel((const void*)attn_stream_kernel, dim3(grid), dim3(kSThreads), smem, pdl, stream, &a);
}
