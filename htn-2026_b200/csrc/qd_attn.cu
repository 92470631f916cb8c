// Split-K GQA flash-decode with log-sum-exp merge, sm_100a.
//
// Grid (splits, kv_heads, batch), 4 warps per CTA. A CTA owns one KV head of one sequence and one
// contiguous key range (chunk) of the static cache; it serves the GROUP = 4 query heads of that KV
// head, so each K/V row is read from HBM once per step. The valid length (pos + 1) is read on the
// device, so one captured launch serves every decode step; keys at or beyond it are never read.
//
// Per warp, 32 keys at a time: lane j computes the four scores of key j (fp32 dot over 128 dims,
// BF16 inputs), the warp updates its running max / sum with fp32 probabilities, rounds them to BF16
// and accumulates P.V with lane j holding dims 4j..4j+3 (the flash-attention arithmetic the
// reference's SDPA and Triton kernels follow, engine/kernels/decode_attn.py:1-11). The four warps'
// states are merged in shared memory, the CTA writes (acc, max, sum) for its split, and the last
// split to arrive (atomic ticket) merges all splits in split order:
//   w_s = exp(m_s - max_s m_s), out = sum_s acc_s w_s / sum_s l_s w_s  (engine/kernels/decode_attn.py:73-86).
#include "qd_common.cuh"
#include "qd_host.h"

namespace qd {

constexpr int kAttnWarps = 4;
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
};

__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
  __shared__ float qs[kGroup][kHeadDim];
  __shared__ float wacc[kAttnWarps][kGroup][kHeadDim];
  __shared__ float wm[kAttnWarps][kGroup], wl[kAttnWarps][kGroup];
  __shared__ int last_flag;

  grid_dep_wait();
  grid_dep_launch();

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int64_t len = ld_cg_s64(a.pos) + 1;
  if (len < 1 || len > a.cap) {  // a position outside the cache: read nothing beyond it, flag it
    if (tid == 0 && split == 0 && a.err) atomicOr(a.err, QD_DEVERR_POS);
    len = len < 1 ? 1 : a.cap;
  }
  const int64_t start = (int64_t)split * a.chunk;
  int64_t end = start + a.chunk;
  if (end > len) end = len;

  for (int h = 0; h < kGroup; ++h) {
    const __nv_bfloat16* qp = a.q + ((int64_t)b * a.nq + kvh * kGroup + h) * kHeadDim;
    const uint16_t u = __ldcg(reinterpret_cast<const unsigned short*>(qp) + tid);
    qs[h][tid] = __uint_as_float((uint32_t)u << 16);
  }
  __syncthreads();

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

  for (int64_t t0 = start + warp * 32; t0 < end; t0 += kAttnWarps * 32) {
    const int64_t key = t0 + lane;
    const bool valid = key < end;
    float s[kGroup] = {0.f, 0.f, 0.f, 0.f};
    if (valid) {
      const __nv_bfloat16* kp = kbase + key * kHeadDim;
#pragma unroll 4
      for (int cq = 0; cq < kHeadDim / 8; ++cq) {
        const uint4 u = ld_cg_v4(kp + cq * 8);
        const float kf[8] = {bf_lo(u.x), bf_hi(u.x), bf_lo(u.y), bf_hi(u.y),
                             bf_lo(u.z), bf_hi(u.z), bf_lo(u.w), bf_hi(u.w)};
#pragma unroll
        for (int h = 0; h < kGroup; ++h)
#pragma unroll
          for (int e = 0; e < 8; ++e) s[h] = fmaf(qs[h][cq * 8 + e], kf[e], s[h]);
      }
    }
    float pb[kGroup];
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      const float sc = valid ? s[h] * a.scale : -INFINITY;
      const float m_new = fmaxf(m_run[h], warp_max(sc));
      const float alpha = expf(m_run[h] - m_new);  // exp(-inf) = 0 on the first tile
      const float p = valid ? expf(sc - m_new) : 0.f;
      l_run[h] = l_run[h] * alpha + warp_sum(p);
#pragma unroll
      for (int d = 0; d < 4; ++d) acc[h][d] *= alpha;
      m_run[h] = m_new;
      pb[h] = bf16r(p);
    }
    const int nk = (int)((end - t0) < 32 ? (end - t0) : 32);
    for (int j = 0; j < nk; ++j) {
      const uint2 u = ld_cg_v2(vbase + (t0 + j) * kHeadDim + 4 * lane);
      const float vf[4] = {bf_lo(u.x), bf_hi(u.x), bf_lo(u.y), bf_hi(u.y)};
#pragma unroll
      for (int h = 0; h < kGroup; ++h) {
        const float pj = __shfl_sync(0xffffffffu, pb[h], j);
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[h][d] = fmaf(pj, vf[d], acc[h][d]);
      }
    }
  }

  // merge the four warps of this CTA
#pragma unroll
  for (int h = 0; h < kGroup; ++h) {
#pragma unroll
    for (int d = 0; d < 4; ++d) wacc[warp][h][4 * lane + d] = acc[h][d];
    if (lane == 0) {
      wm[warp][h] = m_run[h];
      wl[warp][h] = l_run[h];
    }
  }
  __syncthreads();
  const int64_t row0 = ((int64_t)b * a.nq + kvh * kGroup) * a.splits;
  for (int h = 0; h < kGroup; ++h) {
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, wm[w][h]);
    float num = 0.f, den = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        if (wm[w][h] == -INFINITY) continue;
        const float sc = expf(wm[w][h] - mx);
        num = fmaf(wacc[w][h][tid], sc, num);
        den = fmaf(wl[w][h], sc, den);
      }
    }
    const int64_t part = row0 + (int64_t)h * a.splits + split;
    a.part_acc[part * kHeadDim + tid] = num;
    if (tid == 0) {
      a.part_ml[part * 2] = mx;
      a.part_ml[part * 2 + 1] = den;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last_flag = (atomicAdd(a.tickets + (int64_t)b * a.nkv + kvh, 1) == a.splits - 1) ? 1 : 0;
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  for (int h = 0; h < kGroup; ++h) {
    const int64_t prow = row0 + (int64_t)h * a.splits;
    float mx = -INFINITY;
    for (int s = 0; s < a.splits; ++s) mx = fmaxf(mx, ld_cg_f32(a.part_ml + (prow + s) * 2));
    float num = 0.f, den = 0.f;
    for (int s = 0; s < a.splits; ++s) {
      const float ms = ld_cg_f32(a.part_ml + (prow + s) * 2);
      if (ms == -INFINITY) continue;
      const float w = expf(ms - mx);
      num = fmaf(ld_cg_f32(a.part_acc + (prow + s) * kHeadDim + tid), w, num);
      den = fmaf(ld_cg_f32(a.part_ml + (prow + s) * 2 + 1), w, den);
    }
    a.out[((int64_t)b * a.nq + kvh * kGroup + h) * kHeadDim + tid] = __float2bfloat16_rn(num / den);
  }
  if (tid == 0) atomicExch(a.tickets + (int64_t)b * a.nkv + kvh, 0);
}

struct AttnPlan {
  int splits;
  int64_t chunk, off_acc, off_ml, off_tickets, bytes;
};

static bool attn_plan(int batch, int nkv, int64_t cap, int grid_hint, AttnPlan* p) {
  if (batch < 1 || nkv < 1 || cap < 1) return false;
  const int target = grid_hint > 0 ? grid_hint : 2 * host_sm_count();
  int64_t splits = (target + (int64_t)batch * nkv - 1) / ((int64_t)batch * nkv);
  const int64_t max_splits = (cap + 63) / 64;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  int64_t chunk = (cap + splits - 1) / splits;
  chunk = (chunk + 31) / 32 * 32;
  splits = (cap + chunk - 1) / chunk;
  p->splits = (int)splits;
  p->chunk = chunk;
  const int64_t rows = (int64_t)batch * nkv * kGroup * splits;
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  p->off_acc = take(rows * kHeadDim * 4);
  p->off_ml = take(rows * 2 * 4);
  p->off_tickets = take((int64_t)batch * nkv * 4);
  p->bytes = off;
  return true;
}

}  // namespace qd

using namespace qd;

extern "C" int qd_attn_plan(int batch, int nkv_heads, int64_t cap, int grid_hint, int* splits, int64_t* chunk,
                            int64_t* scratch_bytes) {
  AttnPlan p;
  if (!attn_plan(batch, nkv_heads, cap, grid_hint, &p)) return set_error(QD_ERR_ARG, "attn plan: bad sizes");
  if (splits) *splits = p.splits;
  if (chunk) *chunk = p.chunk;
  if (scratch_bytes) *scratch_bytes = p.bytes;
  return QD_OK;
}

extern "C" int qd_attn_decode(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos, void* out,
                              int batch, int nq_heads, int nkv_heads, int64_t cap, int64_t cs_b, int64_t cs_h,
                              int splits, int64_t chunk, float scale, void* scratch, int64_t scratch_bytes, int* err,
                              int pdl, cudaStream_t stream) {
  if (!q || !k_cache || !v_cache || !pos || !out || !scratch) return set_error(QD_ERR_ARG, "null pointer");
  if (nkv_heads < 1 || nq_heads != nkv_heads * kGroup)
    return set_error(QD_ERR_UNSUPPORTED, "attention is built for %d query heads per KV head", kGroup);
  if (batch < 1 || splits < 1 || chunk < 1 || (int64_t)splits * chunk < cap)
    return set_error(QD_ERR_ARG, "splits * chunk must cover the cache capacity");
  if (!aligned16(k_cache) || !aligned16(v_cache) || cs_h < cap * kHeadDim || cs_b < (int64_t)nkv_heads * cs_h ||
      cs_h % 8 || cs_b % 8)
    return set_error(QD_ERR_ARG, "cache strides/alignment");
  if (batch > 65535 || nkv_heads > 65535) return set_error(QD_ERR_UNSUPPORTED, "grid too large");
  const int64_t rows = (int64_t)batch * nq_heads * splits;
  const int64_t need_acc = (rows * kHeadDim * 4 + 255) / 256 * 256, need_ml = (rows * 8 + 255) / 256 * 256;
  const int64_t need = need_acc + need_ml + ((int64_t)batch * nkv_heads * 4 + 255) / 256 * 256;
  if (scratch_bytes < need)
    return set_error(QD_ERR_SCRATCH, "scratch %lld B < %lld B", (long long)scratch_bytes, (long long)need);
  AttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k_cache);
  a.v = static_cast<const __nv_bfloat16*>(v_cache);
  a.pos = pos;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.batch = batch;
  a.nq = nq_heads;
  a.nkv = nkv_heads;
  a.splits = splits;
  a.cap = cap;
  a.cs_b = cs_b;
  a.cs_h = cs_h;
  a.chunk = chunk;
  a.scale = scale;
  char* sc = static_cast<char*>(scratch);
  a.part_acc = reinterpret_cast<float*>(sc);
  a.part_ml = reinterpret_cast<float*>(sc + need_acc);
  a.tickets = reinterpret_cast<int*>(sc + need_acc + need_ml);
  a.err = err;
  return launch_kernel((const void*)attn_decode_kernel, dim3(splits, nkv_heads, batch), dim3(kAttnWarps * 32), 0, pdl,
                       stream, &a);
}
