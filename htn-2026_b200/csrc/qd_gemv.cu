// Streaming BF16 GEMV / skinny GEMM (m <= 8 rows) for the decode step, sm_100a: one launch per
// projection. The device code (stream-K partition, TMA ring, split-K tickets, fused epilogues) is in
// qd_gemv_dev.cuh, shared with the persistent decode-step kernel.
//
// Launched with programmatic dependent launch: the producer warp starts streaming weights (which no
// kernel writes) before the preceding kernel has finished; consumers wait for it before touching
// activations.

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "qd_gemv_dev.cuh"
#include "qd_plan.h"

namespace qd {

struct SmemLayout {
  int ring, xs, red, wsum, lmv, lmi, flags, aux, bars, total;
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
  L.aux = off;
  off += 512 * 4;
  L.bars = align_up(off, 8);
  off = L.bars + 2 * nst * 8;
  L.total = align_up(off, 128);
  return L;
}

template <int M, int MODE>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(1024) char smem[];
  const SmemLayout L = smem_layout(M, a.k, a.nst);
  const Ring R{smem + L.ring, smem_u32(smem + L.bars), a.nst};
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + L.xs);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* wsum = reinterpret_cast<float*>(smem + L.wsum);
  float* lmv = reinterpret_cast<float*>(smem + L.lmv);
  int* lmi = reinterpret_cast<int*>(smem + L.lmi);
  int* flags = reinterpret_cast<int*>(smem + L.flags);
  float* aux = reinterpret_cast<float*>(smem + L.aux);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  if (tid == 0) {
    ring_init(R);
    flags[0] = 0;  // blocks issued by the producer
    flags[1] = 0;  // ticket result broadcast
  }
  if (tid < M) {
    lmv[tid] = -INFINITY;
    lmi[tid] = 0x7fffffff;
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    if (lane == 0) {  // producer: this CTA's contiguous range of weight blocks
      const int64_t b0 = part_begin(a.total, a.grid, cta), b1 = part_begin(a.total, a.grid, cta + 1);
      int slot = 0, round = 0, issued = 0;
      produce_range_prefetch(R, slot, round, issued, a.w + b0 * (int64_t)kBlockBytes, b1 - b0, a.prefetch,
                             policy_evict_first(), a.err);
      flags[0] = issued;
    }
  } else {
    grid_dep_wait();
    grid_dep_launch();
    stage_x<M>(a, xs, wsum, tid);
    int slot = 0, phase = 0;
    bool ok = true;
    consume_blocks<M, MODE>(a, R, slot, phase, cta, xs, red, wsum, lmv, lmi, flags, aux, tid, ok);
    if constexpr (MODE == MODE_LM) lm_global_argmax<M>(a, cta, wsum, lmv, lmi, flags, tid);
  }
  __syncthreads();
  if (tid == 0) ring_drain(R, flags[0], a.err);
}

// ------------------------------------------------------------------ host side

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

// Tuning: QD_GEMV_CTAS_PER_SM CTAs per SM in the grid (default 1), QD_GEMV_STAGES ring depth in 16 KiB
// blocks (default 4), reduced until the CTA's shared memory fits its share of the SM.
static int ctas_per_sm() {
  const int c = env_int("QD_GEMV_CTAS_PER_SM", 1);
  return c < 1 ? 1 : (c > 4 ? 4 : c);
}

// QD_PREFETCH_BLOCKS: blocks each CTA keeps prefetched into L2 beyond its ring (default 8).
int prefetch_blocks() {
  const int v = env_int("QD_PREFETCH_BLOCKS", 8);
  return v < 0 ? 0 : (v > 256 ? 256 : v);
}

static int default_nst(int M, int64_t k) {
  const int fixed = smem_layout(M, k, 0).total;
  const int budget = (ctas_per_sm() == 1 ? 227 * 1024 : 228 * 1024 / ctas_per_sm() - 1024);
  int nst = env_int("QD_GEMV_STAGES", 4);
  if (nst > 16) nst = 16;
  while (nst > 2 && fixed + nst * kBlockBytes + 16 * nst > budget) --nst;
  return nst < 2 ? 2 : nst;
}

int stream_k_smax(int64_t groups, int kblocks, int grid) {
  const int64_t total = groups * kblocks;
  int smax = 1;
  for (int64_t gi = 0; gi < groups; ++gi) {
    const int lo = part_owner(total, grid, gi * kblocks), hi = part_owner(total, grid, gi * kblocks + kblocks - 1);
    if (hi - lo + 1 > smax) smax = hi - lo + 1;
  }
  return smax;
}

bool make_plan(int64_t n_rows, int64_t k, int M, int grid_hint, Plan* p) {
  if (n_rows <= 0 || k <= 0 || n_rows % kBlockRows || k % kBlockCols || M < 1 || M > 8) return false;
  const int kblocks = (int)(k / kBlockCols);
  p->groups = n_rows / kBlockRows;
  p->total = p->groups * kblocks;
  int g = grid_hint > 0 ? grid_hint : host_sm_count() * ctas_per_sm();
  if (g > p->total) g = (int)p->total;
  if (g < 1) g = 1;
  p->grid = g;
  const int smax = stream_k_smax(p->groups, kblocks, g);
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
  if (int rc = set_max_dynamic_smem((const void*)kern, smem)) return rc;
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
  a.prefetch = prefetch_blocks();
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  char* sc = static_cast<char*>(scratch);
  a.tickets = reinterpret_cast<int*>(sc + p.off_tickets);
  a.lm_ticket = reinterpret_cast<int*>(sc + p.off_lm_ticket);
  a.cta_val = reinterpret_cast<float*>(sc + p.off_cta_val);
  a.cta_idx = reinterpret_cast<int*>(sc + p.off_cta_idx);
  a.partials = reinterpret_cast<float*>(sc + p.off_partials);
  a.smax = p.smax;
  a.m_act = M;
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
  // residual projections sum their split-K partials in fixed point, as the persistent step does, so the
  // two paths give the same bits
  a.fx_numerics = mode == MODE_RES ? 1 : 0;
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
  a.fx_numerics = 1;  // fixed-point split-K sums, as the persistent step's deferred QKV
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
