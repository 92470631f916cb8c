// Token-tree verification kernels, sm_100a: attention of the T nodes of a draft tree over the cached
// prefix and their own ancestors, and the compaction of the accepted path's keys / values.
//
// A verify forward runs the T nodes of one token tree per sequence (node 0 = the sequence's last emitted
// token, parents before children) as B x T activation rows, row b * T + i = node i of sequence b.
// Node i's keys / values go to slot prefix[b] + i of its sequence's cache and are rotated at position
// prefix[b] + depth(i) (qd_tree_qk_rope). Node i attends to every cached key [0, prefix[b]) and to the
// tree slots of its ancestors and itself: anc[row] bit j set <=> node j is node i or one of its
// ancestors. Once the accepted paths are known, the keys / values of their nodes move from their tree
// slots to the consecutive slots prefix + depth, where the next step expects them (qd_tree_compact);
// their rotation already used that position. The prefixes live in device memory, so one recorded or
// captured verify serves every round.
#include "qd_common.cuh"
#include "qd_host.h"

namespace qd {

constexpr int kTreeWarps = 4;
constexpr int kTreeThreads = kTreeWarps * 32;
constexpr int kTreeGroup = 4;  // query heads per KV head
constexpr int kHeadDimTree = 128;

struct TreeAttnArgs {
  const __nv_bfloat16* q;  // [B * T, nq * 128], row stride ldq
  const __nv_bfloat16 *k, *v;  // [B, nkv, cap, 128], sequence stride cs_b, head stride cs_h
  __nv_bfloat16* out;          // [B * T, nq * 128], row stride ldo
  const uint32_t* anc;         // [B * T] ancestor masks
  const int32_t* prefix;       // [B] cached keys before each sequence's tree (= its root's slot)
  int* err;
  int64_t ldq, ldo, cs_b, cs_h, cap;
  int T, nq;
  float scale;
};

// One CTA of 4 warps per (KV head, tree row): the node's 4 query heads of that KV head attend over the
// visible keys of its sequence, in slot order (virtual key v < prefix + T; slot v is visible when
// v < prefix or the node's mask has bit v - prefix). Each warp takes 8 keys per pass (4 lanes per key for q.k, dims
// 4 lane.. 4 lane + 3 for P.V); fp32 scores and online softmax, probabilities rounded to BF16 before P.V,
// fp32 accumulation, the 4 warps' (max, sum, acc) combined in warp order - the arithmetic of the decode
// attention's units.
__global__ void __launch_bounds__(kTreeThreads) tree_attn_kernel(const __grid_constant__ TreeAttnArgs a) {
  __shared__ float qs[kTreeGroup][kHeadDimTree];
  __shared__ float wacc[kTreeWarps][kTreeGroup][kHeadDimTree];
  __shared__ float wm[kTreeWarps][kTreeGroup], wl[kTreeWarps][kTreeGroup];
  grid_dep_wait();
  grid_dep_launch();
  const int kvh = blockIdx.x, node = blockIdx.y, seq = node / a.T;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, kj = lane >> 2, qd = lane & 3;
  const int64_t prefix = a.prefix[seq];
  if (prefix < 0 || prefix + a.T > a.cap) {  // the tree would reach past the cache: zeros, error flag
    if (tid == 0 && a.err) atomicOr(a.err, QD_DEVERR_POS);
    for (int h = 0; h < kTreeGroup; ++h)
      a.out[node * a.ldo + (int64_t)(kvh * kTreeGroup + h) * kHeadDimTree + tid] = __float2bfloat16_rn(0.f);
    return;
  }
  for (int h = 0; h < kTreeGroup; ++h) {
    const uint16_t u = __ldcg(reinterpret_cast<const unsigned short*>(a.q + node * a.ldq) +
                              (int64_t)(kvh * kTreeGroup + h) * kHeadDimTree + tid);
    qs[h][tid] = __uint_as_float((uint32_t)u << 16);
  }
  __syncthreads();
  const uint32_t mask = a.anc[node];
  const int64_t nv = prefix + a.T;
  const __nv_bfloat16* kbase = a.k + seq * a.cs_b + (int64_t)kvh * a.cs_h;
  const __nv_bfloat16* vbase = a.v + seq * a.cs_b + (int64_t)kvh * a.cs_h;
  auto visible = [&](int64_t v) { return v < prefix || (v < nv && ((mask >> (int)(v - prefix)) & 1u)); };
  float m_run[kTreeGroup], l_run[kTreeGroup], acc[kTreeGroup][4];
#pragma unroll
  for (int h = 0; h < kTreeGroup; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.f;
#pragma unroll
    for (int d = 0; d < 4; ++d) acc[h][d] = 0.f;
  }
  for (int64_t t0 = warp * 8; t0 < nv; t0 += kTreeWarps * 8) {
    const int64_t key = t0 + kj;
    const bool valid = key < nv && visible(key);
    uint4 kr[4];
    const __nv_bfloat16* kp = kbase + (key < nv ? key : t0) * kHeadDimTree + qd * 32;
#pragma unroll
    for (int c = 0; c < 4; ++c) kr[c] = ld_cg_v4(kp + c * 8);
    uint2 vr[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      vr[j] = (t0 + j < nv && visible(t0 + j)) ? ld_cg_v2(vbase + (t0 + j) * kHeadDimTree + 4 * lane) : make_uint2(0u, 0u);
    float s[kTreeGroup] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float kf[8] = {bf_lo(kr[c].x), bf_hi(kr[c].x), bf_lo(kr[c].y), bf_hi(kr[c].y),
                           bf_lo(kr[c].z), bf_hi(kr[c].z), bf_lo(kr[c].w), bf_hi(kr[c].w)};
#pragma unroll
      for (int h = 0; h < kTreeGroup; ++h)
#pragma unroll
        for (int e = 0; e < 8; ++e) s[h] = fmaf(qs[h][qd * 32 + c * 8 + e], kf[e], s[h]);
    }
    float pb[kTreeGroup];
#pragma unroll
    for (int h = 0; h < kTreeGroup; ++h) {
      s[h] += __shfl_xor_sync(0xffffffffu, s[h], 1);  // the 4 quarters of key kj
      s[h] += __shfl_xor_sync(0xffffffffu, s[h], 2);
      const float sc = valid ? s[h] * a.scale : -INFINITY;
      float mt = sc;
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
      const float m_new = fmaxf(m_run[h], mt);
      // no visible key yet in this warp: nothing to rescale or add
      const float alpha = m_new == -INFINITY ? 1.f : expf(m_run[h] - m_new);
      const float p = valid ? expf(sc - m_new) : 0.f;
      float ps = p;
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
      for (int h = 0; h < kTreeGroup; ++h) {
        const float pj = __shfl_sync(0xffffffffu, pb[h], j * 4);  // 0 for keys that are not visible
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[h][d] = fmaf(pj, vf[d], acc[h][d]);
      }
    }
  }
#pragma unroll
  for (int h = 0; h < kTreeGroup; ++h) {
#pragma unroll
    for (int d = 0; d < 4; ++d) wacc[warp][h][4 * lane + d] = acc[h][d];
    if (lane == 0) {
      wm[warp][h] = m_run[h];
      wl[warp][h] = l_run[h];
    }
  }
  __syncthreads();
  for (int h = 0; h < kTreeGroup; ++h) {
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kTreeWarps; ++w) mx = fmaxf(mx, wm[w][h]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < kTreeWarps; ++w) {
      if (wm[w][h] == -INFINITY) continue;  // a warp that saw no visible key
      const float sc = expf(wm[w][h] - mx);
      num = fmaf(wacc[w][h][tid], sc, num);
      den = fmaf(wl[w][h], sc, den);
    }
    a.out[node * a.ldo + (int64_t)(kvh * kTreeGroup + h) * kHeadDimTree + tid] = __float2bfloat16_rn(num / den);
  }
}

struct TreeCompactArgs {
  __nv_bfloat16 *k, *v;   // [layers][B][nkv][cap][128]
  int64_t layer_stride, cs_b, cs_h;
  const int32_t* moves;  // [n][3]: sequence, source slot, destination slot, applied in order
  int n, batch;
  int64_t cap;
};

// One CTA of 128 threads per (layer, KV head): for each move in order, the 128 values of the key and of
// the value at the source slot of the move's sequence are copied to its destination slot.
__global__ void __launch_bounds__(128) tree_compact_kernel(const __grid_constant__ TreeCompactArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t head = (int64_t)blockIdx.y * a.layer_stride + (int64_t)blockIdx.x * a.cs_h;
  for (int i = 0; i < a.n; ++i) {
    const int64_t b = a.moves[3 * i], s0 = a.moves[3 * i + 1], d0 = a.moves[3 * i + 2];
    // outside the batch or the cache: nothing moves (uniform over the CTA, so the barriers stay matched)
    if (b < 0 || b >= a.batch || s0 < 0 || s0 >= a.cap || d0 < 0 || d0 >= a.cap) continue;
    const int64_t base = head + b * a.cs_b;
    const int64_t src = base + s0 * kHeadDimTree + threadIdx.x;
    const int64_t dst = base + d0 * kHeadDimTree + threadIdx.x;
    const __nv_bfloat16 kv = a.k[src], vv = a.v[src];
    __syncthreads();  // every read of this move before any write (a later move may read a slot written here)
    a.k[dst] = kv;
    a.v[dst] = vv;
    __syncthreads();
  }
}

}  // namespace qd

using namespace qd;

extern "C" int qd_tree_attn(const void* q, int64_t ldq, int batch, int T, int nq_heads, int nkv_heads,
                            const void* k_cache, const void* v_cache, int64_t cap, int64_t cs_b, int64_t cs_h,
                            const int32_t* prefix, const uint32_t* anc, float scale, void* out, int64_t ldo, int* err,
                            cudaStream_t stream) {
  if (!q || !k_cache || !v_cache || !prefix || !anc || !out)
    return set_error(QD_ERR_ARG, "tree attention: null pointer");
  if (batch < 1 || T < 1 || T > 32 || (int64_t)batch * T > 65535 || nkv_heads < 1 ||
      nq_heads != kTreeGroup * nkv_heads || T > cap || cs_h < cap * kHeadDimTree ||
      cs_b < (int64_t)nkv_heads * cs_h || ldq < (int64_t)nq_heads * kHeadDimTree ||
      ldo < (int64_t)nq_heads * kHeadDimTree || ldq % 8 || cs_h % 8 || cs_b % 8)
    return set_error(QD_ERR_ARG, "tree attention: bad sizes (1 <= T <= 32, 4 query heads per KV head, T <= cap)");
  if (!aligned16(k_cache) || !aligned16(v_cache)) return set_error(QD_ERR_ARG, "tree attention: cache alignment");
  TreeAttnArgs a = {};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k_cache);
  a.v = static_cast<const __nv_bfloat16*>(v_cache);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.anc = anc;
  a.prefix = prefix;
  a.err = err;
  a.ldq = ldq;
  a.ldo = ldo;
  a.cs_b = cs_b;
  a.cs_h = cs_h;
  a.cap = cap;
  a.T = T;
  a.nq = nq_heads;
  a.scale = scale;
  return launch_kernel((const void*)tree_attn_kernel, dim3(nkv_heads, batch * T), dim3(kTreeThreads), 0, 1, stream,
                       &a);
}

extern "C" int qd_tree_compact(void* k_cache, void* v_cache, int layers, int64_t layer_stride, int batch,
                               int64_t cs_b, int nkv_heads, int64_t cs_h, int64_t cap, const int32_t* moves, int n,
                               cudaStream_t stream) {
  if (n == 0) return QD_OK;
  if (!k_cache || !v_cache || !moves) return set_error(QD_ERR_ARG, "tree compact: null pointer");
  if (layers < 1 || layers > 65535 || batch < 1 || nkv_heads < 1 || n < 0 || n > 4096 || cs_h < cap * kHeadDimTree ||
      cs_b < (int64_t)nkv_heads * cs_h || layer_stride < (int64_t)batch * cs_b)
    return set_error(QD_ERR_ARG, "tree compact: bad sizes");
  TreeCompactArgs a = {};
  a.k = static_cast<__nv_bfloat16*>(k_cache);
  a.v = static_cast<__nv_bfloat16*>(v_cache);
  a.layer_stride = layer_stride;
  a.cs_b = cs_b;
  a.cs_h = cs_h;
  a.moves = moves;
  a.n = n;
  a.batch = batch;
  a.cap = cap;
  return launch_kernel((const void*)tree_compact_kernel, dim3(nkv_heads, layers), dim3(128), 0, 1, stream, &a);
}
