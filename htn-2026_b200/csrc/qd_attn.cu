// Split-K GQA flash-decode with log-sum-exp merge, sm_100a: grid (splits, kv_heads, batch), one
// unit (sequence, KV head, split) per CTA of 4 warps. The device code is in qd_attn_dev.cuh, shared
// with the persistent decode-step kernel.
#include "qd_attn_dev.cuh"
#include "qd_plan.h"

namespace qd {

__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
  __shared__ AttnSmem sm;
  grid_dep_wait();
  grid_dep_launch();
  const int64_t len = attn_len(a, ld_cg_s64(a.pos), threadIdx.x == 0 && blockIdx.x == 0);
  attn_unit(a, blockIdx.z, blockIdx.y, blockIdx.x, threadIdx.x, 1, sm, len);
}

// QD_ATTN_KEYS_PER_SPLIT: keys per split at run time (default 32); the plan's split count is the cap.
int attn_keys_per_split() {
  const int v = env_int("QD_ATTN_KEYS_PER_SPLIT", 32);
  return v < 32 ? 32 : v;
}

bool attn_plan(int batch, int nkv, int64_t cap, int grid_hint, AttnPlan* p) {
  if (batch < 1 || nkv < 1 || cap < 1) return false;
  const int target = grid_hint > 0 ? grid_hint : 2 * host_sm_count();
  int64_t splits = (target + (int64_t)batch * nkv - 1) / ((int64_t)batch * nkv);
  const int64_t max_splits = (cap + 31) / 32;  // a split covers at least one 32-key pass of a team
  if (splits > max_splits) splits = max_splits;
  if (splits > 160) splits = 160;  // the merge stages (max, sum, weight) of 4 heads x splits in 8 KiB
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
  AttnArgs a = {};
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
  a.done = nullptr;
  a.keys_per_split = attn_keys_per_split();
  return launch_kernel((const void*)attn_decode_kernel, dim3(splits, nkv_heads, batch), dim3(kAttnWarps * 32), 0, pdl,
                       stream, &a);
}
