// Persistent whole-decode-step kernel, sm_100a: one launch runs embedding -> layers x [QKV + q/k
// norm + RoPE + KV append, attention, O + residual, gate_up + SwiGLU, down + residual] -> LM head +
// argmax + position advance.
//
// One CTA per SM (cooperative launch, so every CTA is resident). The producer warp streams this
// CTA's share of every projection's weight blocks, op after op and layer after layer, into one deep
// ring of 16 KiB blocks: weights never depend on activations, so HBM keeps streaming the next
// projection while the consumers wait for the current one's inputs. The eight consumer warps walk
// the same op sequence; before each op, one thread waits (bounded) on the completion counter of the
// op that produces its input, e.g. gate_up waits until all 20 row groups of the O projection are
// finalized. Counters are bumped with release semantics by whoever finalizes a row group (a GEMV
// epilogue) or merges a (sequence, KV head) (attention); all cross-CTA activations are read with
// L2 (.cg) loads after an acquire. The per-op arithmetic is exactly the per-projection kernels'
// (qd_gemv_dev.cuh, qd_attn_dev.cuh) with the same stream-K partition and the same attention splits,
// so the two paths produce bit-identical tokens and logits.
//
// Failure handling: every wait is bounded (1 s); a dependency wait that expires sets QD_DEVERR_DEP
// and an abort flag that makes every later wait return at once, so a broken step finishes (with
// garbage) instead of hanging. The host reads the error word and clears the scratch.
#include "qd_attn_dev.cuh"
#include "qd_gemv_dev.cuh"
#include "qd_plan.h"
#include "qd_umma.cuh"

namespace qd {

enum { K_QKV = 0, K_O = 1, K_GU = 2, K_DOWN = 3, K_LM = 4, K_KINDS = 5 };

struct StepArgs {
  const char *w_qkv, *w_o, *w_gu, *w_down, *e;
  int64_t qkv_lb, o_lb, gu_lb, down_lb;  // bytes per layer
  const __nv_bfloat16 *ln1, *ln2, *qn, *kn, *fnorm;
  int L, H, I, nq, nkv;
  int64_t vocab, vocab_rows;
  float eps, scale;
  int64_t* tok;
  int64_t* pos;
  __nv_bfloat16 *x, *q, *attn, *act, *kc, *vc;
  int64_t c_ls, cs_b, cs_h, cap;
  const __nv_bfloat16 *cos, *sin;
  __nv_bfloat16* logits;
  int64_t ld_logits;
  int* err;
  int grid, nst, splits, kmax, prefetch, prefetch_max, evict_first, keys_per_split;
  int xatoms;  // tensor-core consumers: activation atoms (k-blocks) staged per op, at most
  int chains;  // tensor-core consumers: independent accumulators per segment (1, 2, 4 or 8)
  int fold_max;     // attention folded into the QKV epilogue while the valid length is at most this (0: never)
  int* kv_tickets;  // folded attention: QKV row groups finalized per KV head (6 each), reset by the last
  int64_t chunk;
  int smax[K_KINDS];
  int64_t total[K_KINDS];
  int o_merge;       // 1: attention leaves split partials, the O projection's CTAs merge them
  int* counters;
  int* abort_flag;
  int* tickets;
  float* partials;
  float* attn_acc;
  float* attn_ml;
  int* attn_tickets;
  float* cta_val;
  int* cta_idx;
  int* lm_ticket;
  uint64_t* trace;
};

struct StepLayout {
  int ring, xs, red, wsum, lmv, lmi, flags, aux, attn, bars, total;
  int xop, zero, tslot;  // tensor-core consumers only
};

__host__ __device__ inline int sal(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline StepLayout step_layout(int M, int kmax, int nst) {
  StepLayout L;
  int off = 0;
  L.ring = off;
  off += nst * kBlockBytes;
  L.xs = off;
  off = sal(off + M * kmax * 2, 128);
  L.red = off;
  off += M * kBlockRows * 4;
  L.wsum = off;
  off += M * kConsumerWarps * 4 + 64;
  L.lmv = off;
  off += 32;
  L.lmi = off;
  off += 32;
  L.flags = off;
  off += 48;  // [0..3] as in the GEMV kernels, [4..11] the QKV row groups this CTA finalized
  L.aux = off;
  off += 512 * 4;
  L.attn = sal(off, 16);
  static_assert(sizeof(AttnSmem) % 16 == 0, "attention team buffers must stay 16-byte aligned");
  off = L.attn + 2 * (int)sizeof(AttnSmem);
  L.bars = sal(off, 8);
  off = L.bars + 2 * nst * 8;
  L.total = sal(off, 128);
  L.xop = L.zero = L.tslot = -1;
  return L;
}

// Shared memory of the tensor-core variant (offsets from a 1 KiB-aligned base): the weight ring, then
// the B operand of the current projection - `xatoms` 1 KiB atoms, one per k-block the CTA's range
// touches, each 8 rows x 128 B in the 128-byte swizzle with the activation rows 0..M-1 in its first M
// rows and zeros below - and one all-zero atom that stands for operand rows 8..15.
__host__ __device__ inline StepLayout step_mma_layout(int M, int xatoms, int nst) {
  StepLayout L;
  int off = 0;
  L.ring = off;
  off += nst * kBlockBytes;
  L.xop = off;
  off += xatoms * 1024;
  L.zero = off;
  off += 1024;
  L.xs = -1;
  L.red = off;
  off += M * kBlockRows * 4;
  L.wsum = off;
  off += M * kConsumerWarps * 4 + 64;
  L.lmv = off;
  off += 32;
  L.lmi = off;
  off += 32;
  L.flags = off;
  off += 48;  // [0..3] as in the GEMV kernels, [4..11] the QKV row groups this CTA finalized
  L.aux = off;
  off += 512 * 4;
  L.attn = sal(off, 16);
  off = L.attn + 2 * (int)sizeof(AttnSmem);
  L.bars = sal(off, 8);
  off = L.bars + (2 * nst + 5) * 8;  // ring full / empty, accumulator full x2 / empty x2, operand ready
  L.tslot = off;
  off += 16;
  L.total = sal(off, 1024);
  return L;
}

// Optional timeline: trace[(cta * ops + op) * 4 + what], what = 0 input ready, 1 staged, 2 done,
// 3 producer issued the op's last block.
__device__ __forceinline__ void stamp(const StepArgs& A, int cta, int op, int what, int tid) {
  if (A.trace && tid == 0) A.trace[((int64_t)cta * (2 + 5 * A.L) + op) * 4 + what] = globaltimer();
}

// counters: [0] embedding rows; layer l: 1 + 5l + {0 qkv heads, 1 attention merges, 2 o groups,
// 3 gate_up groups, 4 down groups}
__device__ __forceinline__ int* ctr(const StepArgs& A, int l, int op) { return A.counters + 1 + 5 * l + op; }

// One consumer thread waits (bounded) until *cnt >= target, then the 256 consumers proceed.
static __device__ void wait_dep(const StepArgs& A, const int* cnt, int target, int tid) {
  if (tid == 0 && ld_acquire(cnt) < target && !ld_volatile(A.abort_flag)) {
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0;; ++i) {
      if (ld_acquire(cnt) >= target) break;
      if (ld_volatile(A.abort_flag)) break;
      if ((i & 255u) == 255u && globaltimer() - t0 > kWaitLimitNs) {
        atomicOr(A.err, kErrDep);
        atomicExch(A.abort_flag, 1);
        break;
      }
    }
  }
  named_bar(kBarConsumers, kConsumers);
}

// The O projection's input at batch 1..8: attention units leave their split partials (acc, max, sum)
// and each O CTA merges, for the query heads its K-range reads (K-block kb = dims 64kb.. = head kb/2),
// exactly what the attention kernel's last split computes (same order, same operations), into xs.
// Saves the split ticket, the merge's round trips and the output write + reload on the critical path.
// Shared-memory address of activation row m (< 8), k-column kk of the tensor-core B operand: atom
// (kk / 64 - kb_first) mod kblocks, 16-byte chunk (kk % 64) / 8 swizzled with the row.
__device__ __forceinline__ __nv_bfloat16* atom_elem(char* xop, int kblocks, int kb_first, int m, int64_t kk) {
  int s = (int)(kk >> 6) - kb_first;
  if (s < 0) s += kblocks;
  const int c = (int)(kk & 63) >> 3;
  return reinterpret_cast<__nv_bfloat16*>(xop + s * 1024 + m * 128 + ((c ^ m) << 4)) + (kk & 7);
}

// ATOMS = false: the merged heads go to the row-major xs [M][k]; true: to the tensor-core B operand
// atoms of the CTA's k-range (xop, first k-block kb_first), followed by the proxy fence the MMAs need.
template <int M, bool ATOMS>
static __device__ void stage_attn_merge(const StepArgs& A, const GemvArgs& op, int n_use, int cta,
                                        __nv_bfloat16* xs, char* xop, float* scr, int tid) {
  const int64_t b0 = part_begin(op.total, op.grid, cta), b1 = part_begin(op.total, op.grid, cta + 1);
  uint32_t mask = 0;
  int kb = (int)(b0 % op.kblocks);
  for (int64_t b = b0; b < b1; ++b) {
    mask |= 1u << (kb >> 1);
    if (++kb == op.kblocks) kb = 0;
  }
  const int nh = __popc(mask), P = M * nh, E = P * n_use;
  float* mm = scr;  // [P][n_use] maxima, sums, weights; [P] denominators
  float* ll = mm + E;
  float* ww = ll + E;
  float* den = ww + E;
  for (int t = tid; t < E; t += kConsumers) {
    const int p = t / n_use, sp = t - p * n_use, m = p / nh, hq = __fns(mask, 0, p - m * nh + 1);
    const int64_t part = ((int64_t)m * A.nq + hq) * A.splits + sp;
    mm[t] = ld_cg_f32(A.attn_ml + part * 2);
    ll[t] = ld_cg_f32(A.attn_ml + part * 2 + 1);
  }
  named_bar(kBarConsumers, kConsumers);
  for (int t = tid; t < E; t += kConsumers) {
    const int p = t / n_use;
    float mx = -INFINITY;
    for (int sp = 0; sp < n_use; ++sp) mx = fmaxf(mx, mm[p * n_use + sp]);
    ww[t] = (mm[t] == -INFINITY) ? 0.f : expf(mm[t] - mx);
  }
  named_bar(kBarConsumers, kConsumers);
  for (int p = tid; p < P; p += kConsumers) {
    float d = 0.f;
    for (int sp = 0; sp < n_use; ++sp) d = fmaf(ll[p * n_use + sp], ww[p * n_use + sp], d);
    den[p] = d;
  }
  named_bar(kBarConsumers, kConsumers);
  // out = bf16(sum_s acc_s w_s / sum_s l_s w_s) in split order, eight loads in flight at a time
  for (int idx = tid; idx < P * kHeadDim; idx += kConsumers) {
    const int p = idx >> 7, d = idx & 127, m = p / nh, hq = __fns(mask, 0, p - m * nh + 1);
    const int64_t row = ((int64_t)m * A.nq + hq) * A.splits;
    float num = 0.f;
    for (int s0 = 0; s0 < n_use; s0 += 8) {
      float av[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) av[j] = (s0 + j < n_use) ? ld_cg_f32(A.attn_acc + (row + s0 + j) * kHeadDim + d) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (s0 + j < n_use) num = fmaf(av[j], ww[p * n_use + s0 + j], num);
    }
    const __nv_bfloat16 v = __float2bfloat16_rn(num / den[p]);
    if constexpr (ATOMS) {
      // a head's two k-blocks may straddle the range's ends: only the staged atoms are written
      const int64_t kk = (int64_t)hq * kHeadDim + d;
      const int kb_first = (int)(b0 % op.kblocks);
      int sx = (int)(kk >> 6) - kb_first;
      if (sx < 0) sx += op.kblocks;
      if (sx < (b1 - b0 < op.kblocks ? (int)(b1 - b0) : op.kblocks)) *atom_elem(xop, op.kblocks, kb_first, m, kk) = v;
    } else {
      xs[(int64_t)m * op.k + hq * kHeadDim + d] = v;
    }
  }
  if constexpr (ATOMS) fence_proxy_async_smem();
  named_bar(kBarConsumers, kConsumers);
}

// Tensor-core consumers: stage activation rows 0..M-1 of a projection's input (RMSNorm-ed when
// a.norm_w is set, Qwen3RMSNorm's cast placement as in stage_x) into the B operand atoms of the k-blocks
// that this CTA's block range [b0, b1) touches. Rows past the range still enter the sum of squares.
// Ends with the proxy fence and a consumer barrier.
template <int M>
__device__ void stage_atoms(const GemvArgs& a, char* xop, int64_t b0, int64_t b1, float* wsum, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int kv8 = (int)(a.k >> 3);
  const int kb_first = (int)(b0 % a.kblocks);
  const int natoms = (int)(b1 - b0 < a.kblocks ? b1 - b0 : a.kblocks);
  auto needed = [&](int q) {  // chunk q (8 columns) lies in a staged atom
    int s = (q >> 3) - kb_first;
    if (s < 0) s += a.kblocks;
    return s < natoms;
  };
  for (int m = 0; m < M; ++m) {
    float sq = 0.f;
    if (a.norm_w) {  // every chunk feeds the norm; the needed ones are kept
      for (int q0 = 0; q0 < kv8; q0 += kStageBatch * kConsumers) {
        uint4 v[kStageBatch];
#pragma unroll
        for (int j = 0; j < kStageBatch; ++j) {
          const int q = q0 + j * kConsumers + tid;
          v[j] = q < kv8 ? ld_cg_v4(a.x + m * a.ldx + q * 8) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < kStageBatch; ++j) {
          const int q = q0 + j * kConsumers + tid;
          if (q >= kv8) continue;
          const uint32_t u[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = bf_lo(u[e]), hi = bf_hi(u[e]);
            sq = fmaf(lo, lo, sq);
            sq = fmaf(hi, hi, sq);
          }
          if (needed(q)) *reinterpret_cast<uint4*>(atom_elem(xop, a.kblocks, kb_first, m, (int64_t)q * 8)) = v[j];
        }
      }
      sq = warp_sum(sq);
      if (lane == 0) wsum[m * kConsumerWarps + warp] = sq;
    } else {  // no norm: load only the chunks of the staged atoms
      for (int t = tid; t < natoms * 8; t += kConsumers) {
        const int kb = (kb_first + (t >> 3)) % a.kblocks;
        const int q = kb * 8 + (t & 7);
        *reinterpret_cast<uint4*>(atom_elem(xop, a.kblocks, kb_first, m, (int64_t)q * 8)) =
            ld_cg_v4(a.x + m * a.ldx + q * 8);
      }
    }
  }
  named_bar(kBarConsumers, kConsumers);
  if (a.norm_w) {
    for (int m = 0; m < M; ++m) {
      float ss = 0.f;
#pragma unroll
      for (int w8 = 0; w8 < kConsumerWarps; ++w8) ss += wsum[m * kConsumerWarps + w8];
      const float rstd = 1.0f / sqrtf(ss / (float)a.k + a.eps);
      for (int t = tid; t < natoms * 8; t += kConsumers) {
        const int kb = (kb_first + (t >> 3)) % a.kblocks;
        const int q = kb * 8 + (t & 7);
        uint4* p = reinterpret_cast<uint4*>(atom_elem(xop, a.kblocks, kb_first, m, (int64_t)q * 8));
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
  }
  fence_proxy_async_smem();
  named_bar(kBarConsumers, kConsumers);
}

// Tensor-core consumers of one projection: per row-group segment of this CTA's range, wait for the MMA
// warp's accumulator (two alternate, 16 fp32 columns each, at tmem + 16 buf), read rows 0..M-1 of it
// into red (warps 0-3, one TMEM lane quarter each), release it, and run the same split-K flush and
// fused epilogue as the CUDA-core consumers. `buf` / `aph` (accumulator and its phases) carry across
// projections in the MMA warp's order.
template <int M, int MODE>
__device__ void consume_mma(const GemvArgs& a, int cta, uint32_t tmem, int chains, uint32_t accf0, uint32_t acce0,
                            int& buf, int* aph, float* red, float* wsum, float* lmv, int* lmi, int* flags, float* aux,
                            int* abort_flag, int tid, bool& ok) {
  const int warp = tid >> 5, lane = tid & 31;
  if constexpr (MODE == MODE_QKV) qkv_prologue(a, aux, flags, tid);
  const int64_t b_begin = part_begin(a.total, a.grid, cta);
  const int64_t b_end = part_begin(a.total, a.grid, cta + 1);
  int64_t seg_first = b_begin;
  int g = (int)(b_begin / a.kblocks);
  int kb = (int)(b_begin - (int64_t)g * a.kblocks) - 1;
  for (int64_t b = b_begin; b < b_end; ++b) {
    if (++kb == a.kblocks) {
      kb = 0;
      ++g;
    }
    if (!((kb == a.kblocks - 1) || (b == b_end - 1))) continue;
    if (ok) ok = mbar_wait_abort(accf0 + 8u * buf, aph[buf], a.err, kErrWaitFull, abort_flag);
    aph[buf] ^= 1;
    tc_fence_after();
    if (warp < 4) {
      // the segment's MMA k-steps went round-robin to `chains` accumulators; the ones it wrote (4 per
      // block) are summed in chain order
      const int used = (int)(4 * (b - seg_first + 1) < chains ? 4 * (b - seg_first + 1) : chains);
      float sum[M];
#pragma unroll
      for (int m = 0; m < M; ++m) sum[m] = 0.f;
      for (int c = 0; c < used; ++c) {
        float v[M <= 4 ? 4 : 8];
        const uint32_t ta = tmem + ((uint32_t)(32 * warp) << 16) + 16u * (buf * chains + c);
        if constexpr (M <= 4)
          tmem_ld4(ta, v);
        else
          tmem_ld8(ta, v);
        tmem_wait_ld();
#pragma unroll
        for (int m = 0; m < M; ++m) sum[m] = c == 0 ? v[m] : sum[m] + v[m];
      }
#pragma unroll
      for (int m = 0; m < M; ++m) red[m * kBlockRows + 32 * warp + lane] = sum[m];
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8u * buf);
    }
    buf ^= 1;
    named_bar(kBarConsumers, kConsumers);
    flush_segment<M, MODE>(a, g, seg_first, b, cta, red, wsum, lmv, lmi, aux, flags, tid);
    seg_first = b + 1;
  }
}

template <int M>
static __device__ GemvArgs gemv_op(const StepArgs& A, int kind, int l) {
  GemvArgs a = {};
  a.m_act = M;
  a.grid = A.grid;
  a.nst = A.nst;
  a.partials = A.partials;
  a.tickets = A.tickets;
  a.err = A.err;
  a.eps = A.eps;
  a.smax = A.smax[kind];
  a.total = A.total[kind];
  if (kind == K_QKV) {
    a.x = A.x;
    a.ldx = A.H;
    a.k = A.H;
    a.n = (int64_t)(A.nq + 2 * A.nkv) * 128;
    a.w = A.w_qkv + l * A.qkv_lb;
    a.norm_w = A.ln1 + (int64_t)l * A.H;
    a.q_norm = A.qn + l * 128;
    a.k_norm = A.kn + l * 128;
    a.cos = A.cos;
    a.sin = A.sin;
    a.pos = A.pos;
    a.cap = A.cap;
    a.nq = A.nq;
    a.nkv = A.nkv;
    a.q_out = A.q;
    a.k_cache = A.kc + l * A.c_ls;
    a.v_cache = A.vc + l * A.c_ls;
    a.cs_b = A.cs_b;
    a.cs_h = A.cs_h;
    a.done = ctr(A, l, 0);
    a.pos_ready = 1;
  } else if (kind == K_O) {
    a.x = A.attn;
    a.ldx = (int64_t)A.nq * 128;
    a.k = (int64_t)A.nq * 128;
    a.n = A.H;
    a.w = A.w_o + l * A.o_lb;
    a.out = A.x;
    a.ldo = A.H;
    a.res = A.x;
    a.ldr = A.H;
    a.done = ctr(A, l, 2);
  } else if (kind == K_GU) {
    a.x = A.x;
    a.ldx = A.H;
    a.k = A.H;
    a.n = 2 * (int64_t)A.I;
    a.w = A.w_gu + l * A.gu_lb;
    a.norm_w = A.ln2 + (int64_t)l * A.H;
    a.out = A.act;
    a.ldo = A.I;
    a.done = ctr(A, l, 3);
  } else if (kind == K_DOWN) {
    a.x = A.act;
    a.ldx = A.I;
    a.k = A.I;
    a.n = A.H;
    a.w = A.w_down + l * A.down_lb;
    a.out = A.x;
    a.ldo = A.H;
    a.res = A.x;
    a.ldr = A.H;
    a.done = ctr(A, l, 4);
  } else {  // LM head
    a.x = A.x;
    a.ldx = A.H;
    a.k = A.H;
    a.n = A.vocab_rows;
    a.n_valid = A.vocab;
    a.w = A.e;
    a.norm_w = A.fnorm;
    a.tok = A.tok;
    a.pos_inc = A.pos;
    a.inc_pos = 1;
    a.logits = A.logits;
    a.ld_logits = A.ld_logits;
    a.cta_val = A.cta_val;
    a.cta_idx = A.cta_idx;
    a.lm_ticket = A.lm_ticket;
  }
  if (a.n_valid == 0) a.n_valid = a.n;
  a.kblocks = (int)(a.k / kBlockCols);
  return a;
}

// The producer's block sequence: segment 4l + k is this CTA's stream-K range of projection k of layer
// l (k: 0 qkv, 1 o, 2 gate_up, 3 down); segment 4L is its range of the LM head.
struct StepSeg {
  const char* base;
  int64_t n;
};
__device__ constexpr int kOpOfKind[4] = {0, 2, 3, 4};  // position of projection k among a layer's 5 ops

__device__ __forceinline__ StepSeg step_seg(const StepArgs& A, int cta, int s) {
  const int kind = (s == 4 * A.L) ? (int)K_LM : (s & 3);
  const int l = s >> 2;
  const char* base = kind == K_LM ? A.e
                     : kind == K_QKV ? A.w_qkv + l * A.qkv_lb
                     : kind == K_O   ? A.w_o + l * A.o_lb
                     : kind == K_GU  ? A.w_gu + l * A.gu_lb
                                     : A.w_down + l * A.down_lb;
  const int64_t b0 = part_begin(A.total[kind], A.grid, cta), b1 = part_begin(A.total[kind], A.grid, cta + 1);
  return StepSeg{base + b0 * (int64_t)kBlockBytes, b1 - b0};
}

__device__ __forceinline__ int64_t attn_len_of(const StepArgs& A, int64_t pos) {
  AttnArgs t = {};
  t.cap = A.cap;
  return attn_len(t, pos, false);
}
__device__ __forceinline__ int attn_active_of(const StepArgs& A, int64_t len, int64_t* chunk) {
  AttnArgs t = {};
  t.splits = A.splits;
  t.chunk = A.chunk;
  t.keys_per_split = A.keys_per_split;
  return attn_active(t, len, chunk);
}

// Folded attention (short caches): the CTA that finalizes the last of a KV head's six QKV row groups
// (its 4 query heads, key and value) attends, right there, with all 8 consumer warps: every key of
// the valid length for those 4 query heads of every sequence, and writes the final output rows - no
// separate attention phase, no split partials, no merge by the O projection. Same arithmetic as the
// split kernels' units (fp32 scores and online softmax, probabilities rounded to BF16 before P.V, fp32
// accumulation), the 8 warps' (max, sum, acc) combined in warp order. Each warp takes 8 keys per pass
// (the 8 warps cover 64 consecutive keys) and loads the next pass's keys before computing this one.
struct FoldSmem {
  float qs[kGroup][kHeadDim];
  float wacc[kConsumerWarps][kGroup][kHeadDim];
  float wm[kConsumerWarps][kGroup], wl[kConsumerWarps][kGroup];
};

template <int M>
__device__ void attn_fold(const StepArgs& A, int l, int kvh, int64_t len, FoldSmem& sm, int tid) {
  const int warp = tid >> 5, lane = tid & 31, kj = lane >> 2, qd = lane & 3;
  constexpr int kPass = kConsumerWarps * 8;
  for (int m = 0; m < M; ++m) {
    for (int t = tid; t < kGroup * kHeadDim; t += kConsumers) {
      const int h = t >> 7, d = t & 127;
      const uint16_t u = __ldcg(reinterpret_cast<const unsigned short*>(A.q) +
                                ((int64_t)m * A.nq + kvh * kGroup + h) * kHeadDim + d);
      sm.qs[h][d] = __uint_as_float((uint32_t)u << 16);
    }
    named_bar(kBarConsumers, kConsumers);
    const __nv_bfloat16* kbase = A.kc + l * A.c_ls + (int64_t)m * A.cs_b + (int64_t)kvh * A.cs_h;
    const __nv_bfloat16* vbase = A.vc + l * A.c_ls + (int64_t)m * A.cs_b + (int64_t)kvh * A.cs_h;
    float m_run[kGroup], l_run[kGroup], acc[kGroup][4];
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      m_run[h] = -INFINITY;
      l_run[h] = 0.f;
#pragma unroll
      for (int d = 0; d < 4; ++d) acc[h][d] = 0.f;
    }
    uint4 kr[4];
    uint2 vr[8];
    auto load_pass = [&](int64_t t0) {
      const int64_t key = t0 + kj;
      const int nk = (int)((len - t0) < 8 ? (len - t0) : 8);
      const __nv_bfloat16* kp = kbase + (key < len ? key : t0) * kHeadDim + qd * 32;
#pragma unroll
      for (int c = 0; c < 4; ++c) kr[c] = ld_cg_v4(kp + c * 8);
#pragma unroll
      for (int j = 0; j < 8; ++j) vr[j] = (j < nk) ? ld_cg_v2(vbase + (t0 + j) * kHeadDim + 4 * lane) : make_uint2(0u, 0u);
    };
    int64_t t0 = warp * 8;
    if (t0 < len) load_pass(t0);
    for (; t0 < len; t0 += kPass) {
      const uint4 k0 = kr[0], k1 = kr[1], k2 = kr[2], k3 = kr[3];
      uint2 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = vr[j];
      const bool valid = t0 + kj < len;
      if (t0 + kPass < len) load_pass(t0 + kPass);  // in flight while this pass computes
      const uint4 kk[4] = {k0, k1, k2, k3};
      float sc4[kGroup] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float kf[8] = {bf_lo(kk[c].x), bf_hi(kk[c].x), bf_lo(kk[c].y), bf_hi(kk[c].y),
                             bf_lo(kk[c].z), bf_hi(kk[c].z), bf_lo(kk[c].w), bf_hi(kk[c].w)};
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
          const float4 q0 = *reinterpret_cast<const float4*>(&sm.qs[h][qd * 32 + c * 8]);
          const float4 q1 = *reinterpret_cast<const float4*>(&sm.qs[h][qd * 32 + c * 8 + 4]);
          sc4[h] = fmaf(q0.x, kf[0], sc4[h]);
          sc4[h] = fmaf(q0.y, kf[1], sc4[h]);
          sc4[h] = fmaf(q0.z, kf[2], sc4[h]);
          sc4[h] = fmaf(q0.w, kf[3], sc4[h]);
          sc4[h] = fmaf(q1.x, kf[4], sc4[h]);
          sc4[h] = fmaf(q1.y, kf[5], sc4[h]);
          sc4[h] = fmaf(q1.z, kf[6], sc4[h]);
          sc4[h] = fmaf(q1.w, kf[7], sc4[h]);
        }
      }
      float pb[kGroup];
#pragma unroll
      for (int h = 0; h < kGroup; ++h) {
        float sv = sc4[h];
        sv += __shfl_xor_sync(0xffffffffu, sv, 1);  // the 4 quarters of key kj
        sv += __shfl_xor_sync(0xffffffffu, sv, 2);
        const float sc = valid ? sv * A.scale : -INFINITY;
        float mt = sc;  // the 4 lanes of a key agree: reduce over the warp's 8 keys
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
        const float m_new = fmaxf(m_run[h], mt);
        const float alpha = expf(m_run[h] - m_new);
        const float pr = valid ? expf(sc - m_new) : 0.f;
        float ps = pr;
        ps += __shfl_xor_sync(0xffffffffu, ps, 4);
        ps += __shfl_xor_sync(0xffffffffu, ps, 8);
        ps += __shfl_xor_sync(0xffffffffu, ps, 16);
        l_run[h] = l_run[h] * alpha + ps;
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[h][d] *= alpha;
        m_run[h] = m_new;
        pb[h] = bf16r(pr);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float vf[4] = {bf_lo(v[j].x), bf_hi(v[j].x), bf_lo(v[j].y), bf_hi(v[j].y)};
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
          const float pj = __shfl_sync(0xffffffffu, pb[h], j * 4);  // 0 for keys past the end
#pragma unroll
          for (int d = 0; d < 4; ++d) acc[h][d] = fmaf(pj, vf[d], acc[h][d]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
#pragma unroll
      for (int d = 0; d < 4; ++d) sm.wacc[warp][h][4 * lane + d] = acc[h][d];
      if (lane == 0) {
        sm.wm[warp][h] = m_run[h];
        sm.wl[warp][h] = l_run[h];
      }
    }
    named_bar(kBarConsumers, kConsumers);
    for (int t = tid; t < kGroup * kHeadDim; t += kConsumers) {
      const int h = t >> 7, d = t & 127;
      float mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) mx = fmaxf(mx, sm.wm[w][h]);
      float num = 0.f, den = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        if (sm.wm[w][h] == -INFINITY) continue;  // a warp that saw no key
        const float sc = expf(sm.wm[w][h] - mx);
        num = fmaf(sm.wacc[w][h][d], sc, num);
        den = fmaf(sm.wl[w][h], sc, den);
      }
      A.attn[((int64_t)m * A.nq + kvh * kGroup + h) * kHeadDim + d] = __float2bfloat16_rn(num / den);
    }
    named_bar(kBarConsumers, kConsumers);  // shared memory is reused by the next sequence
  }
}

// After the QKV projection of layer l: for every row group this CTA finalized, count it on its KV
// head's ticket; the CTA that completes a KV head (6 groups) runs that head's folded attention, resets
// the ticket and signals the attention counter.
template <int M>
__device__ void fold_after_qkv(const StepArgs& A, int cta, int l, int64_t len, int* fin, int* flags, FoldSmem& sm,
                               int tid) {
  const int n = fin[0];
  for (int i = 0; i < n; ++i) {
    const int g = fin[1 + i];
    const int kvh = g < A.nq ? g / kGroup : (g < A.nq + A.nkv ? g - A.nq : g - A.nq - A.nkv);
    if (tid == 0) flags[1] = (atom_add_acq_rel(A.kv_tickets + kvh, 1) == kGroup + 1) ? 1 : 0;
    named_bar(kBarConsumers, kConsumers);
    if (flags[1]) {  // timeline: the attention op's stamps 0 / 2 bracket the folded attention
      stamp(A, cta, 2 + 5 * l, 0, tid);
      attn_fold<M>(A, l, kvh, len, sm, tid);
      stamp(A, cta, 2 + 5 * l, 2, tid);
      if (tid == 0) atomicExch(A.kv_tickets + kvh, 0);
      signal_done(ctr(A, l, 1), tid);
    }
    named_bar(kBarConsumers, kConsumers);
  }
  if (tid == 0) fin[0] = 0;
  named_bar(kBarConsumers, kConsumers);
}

// Stage a projection's input for the consumers of either variant: row-major xs for the CUDA-core
// consumers; the B operand atoms plus the operand-ready signal for the MMA warp otherwise.
template <int M, bool MMA>
__device__ __forceinline__ void step_stage(const GemvArgs& op, int cta, __nv_bfloat16* xs, char* xop, uint32_t xready,
                                           float* wsum, int tid) {
  if constexpr (MMA) {
    stage_atoms<M>(op, xop, part_begin(op.total, op.grid, cta), part_begin(op.total, op.grid, cta + 1), wsum, tid);
    if (tid == 0) mbar_arrive(xready);
  } else {
    stage_x<M>(op, xs, wsum, tid);
  }
}

template <int M, int MODE, bool MMA>
__device__ __forceinline__ void step_consume(const GemvArgs& op, const Ring& R, int& slot, int& phase, int cta,
                                             const __nv_bfloat16* xs, uint32_t tmem, int chains, uint32_t accf0,
                                             uint32_t acce0,
                                             int& abuf, int* aph, float* red, float* wsum, float* lmv, int* lmi,
                                             int* flags, float* aux, int* abort_flag, int tid, bool& ok) {
  if constexpr (MMA)
    consume_mma<M, MODE>(op, cta, tmem, chains, accf0, acce0, abuf, aph, red, wsum, lmv, lmi, flags, aux, abort_flag,
                         tid, ok);
  else
    consume_blocks<M, MODE>(op, R, slot, phase, cta, xs, red, wsum, lmv, lmi, flags, aux, tid, ok);
}

// MMA = false: eight consumer warps multiply the weight blocks on the CUDA cores (288 threads).
// MMA = true: warp 9 issues the projections as tcgen05 MMAs - swap-AB, M = 128 weight rows of a packed
// block (the A operand as the ring holds it), N = 16 (activation rows 0..M-1 staged by the consumers in
// the B operand atoms, rows M..15 zero), K = 16 per instruction, 4 per block - into two alternating
// 16-column accumulators in tensor memory; the consumers stage operands, read accumulators and run the
// same flushes, epilogues and attention (320 threads). Both run the same ops, partitions and counters.
template <int M, bool MMA>
__global__ void __launch_bounds__(MMA ? kThreads + 32 : kThreads, 1) step_kernel(const __grid_constant__ StepArgs A) {
  extern __shared__ __align__(1024) char smem_raw[];
  // operand atoms use the 128-byte swizzle, a function of the shared address: 1 KiB-aligned base
  char* smem = MMA ? smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u) : smem_raw;
  const StepLayout Ly = MMA ? step_mma_layout(M, A.xatoms, A.nst) : step_layout(M, A.kmax, A.nst);
  const Ring R{smem + Ly.ring, smem_u32(smem + Ly.bars), A.nst};
  __nv_bfloat16* xs = MMA ? nullptr : reinterpret_cast<__nv_bfloat16*>(smem + Ly.xs);
  char* xop = MMA ? smem + Ly.xop : nullptr;
  const uint32_t accf0 = smem_u32(smem + Ly.bars) + 16u * A.nst;  // MMA: accumulator full x2, empty x2, ready
  const uint32_t acce0 = accf0 + 16u, xready = accf0 + 32u;
  uint32_t* tslot = MMA ? reinterpret_cast<uint32_t*>(smem + Ly.tslot) : nullptr;
  float* red = reinterpret_cast<float*>(smem + Ly.red);
  float* wsum = reinterpret_cast<float*>(smem + Ly.wsum);
  float* lmv = reinterpret_cast<float*>(smem + Ly.lmv);
  int* lmi = reinterpret_cast<int*>(smem + Ly.lmi);
  int* flags = reinterpret_cast<int*>(smem + Ly.flags);
  float* aux = reinterpret_cast<float*>(smem + Ly.aux);
  AttnSmem* asm_team = reinterpret_cast<AttnSmem*>(smem + Ly.attn);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  const int G = A.grid;
  if (tid == 0) {
    if constexpr (MMA) {  // ring slots are released by the MMA warp's commits
      for (int st = 0; st < A.nst; ++st) {
        mbar_init(R.full(st), 1);
        mbar_init(R.empty(st), 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(accf0 + 8u * i, 1);
        mbar_init(acce0 + 8u * i, 4);  // consumer warps 0-3 read the accumulator
      }
      mbar_init(xready, 1);
      fence_mbar_init();
    } else {
      ring_init(R);
    }
    flags[0] = 0;
    flags[1] = 0;
  }
  if (tid < M) {
    lmv[tid] = -INFINITY;
    lmi[tid] = 0x7fffffff;
  }
  if constexpr (MMA) {
    if (warp < kConsumerWarps) {  // operand atoms and the zero atom start (and rows >= M stay) zero
      uint4* z = reinterpret_cast<uint4*>(xop);
      for (int i = tid; i < (A.xatoms + 1) * 64; i += kConsumers) z[i] = make_uint4(0u, 0u, 0u, 0u);
      fence_proxy_async_smem();
    }
    if (warp == kConsumerWarps + 1) tmem_alloc(smem_u32(tslot), 256);  // the MMA warp owns the accumulators
    tc_fence_before();
  }
  __syncthreads();
  if constexpr (MMA) tc_fence_after();
  const uint32_t tmem = MMA ? *tslot : 0u;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer: every weight block, in op order
    if (lane == 0) {
      const uint64_t pol = A.evict_first ? policy_evict_first() : policy_evict_normal();
      int slot = 0, round = 0, issued = 0;
      const int nseg = 4 * A.L + 1;  // layer l kind k = segment 4l + k; the LM head last
      int ps = 0;                    // L2 prefetch cursor: segment, block, blocks prefetched so far
      int64_t po = 0, pf_count = 0;
      StepSeg pseg = step_seg(A, cta, 0);
      bool ok = true;
      for (int sgi = 0; sgi < nseg && ok; ++sgi) {
        const StepSeg sg = step_seg(A, cta, sgi);
        for (int64_t i = 0; i < sg.n; ++i) {
          // L2 lookahead: at least `prefetch` blocks beyond the next copy; while the ring is full (the
          // consumers are busy with a dependency, an epilogue or attention) grow it up to
          // `prefetch_max` blocks so HBM keeps streaming through the stall
          auto prefetch_one = [&]() -> bool {
            while (ps < nseg && po >= pseg.n) {
              if (++ps < nseg) pseg = step_seg(A, cta, ps);
              po = 0;
            }
            if (ps >= nseg) return false;
            prefetch_l2(pseg.base + po * (int64_t)kBlockBytes, kBlockBytes);
            ++po;
            ++pf_count;
            return true;
          };
          while (pf_count <= (int64_t)issued + A.prefetch && prefetch_one()) {
          }
          if (round > 0) {
            const uint32_t par = (round - 1) & 1;
            while (!mbar_try_wait(R.empty(slot), par)) {
              if (pf_count > (int64_t)issued + A.prefetch_max || !prefetch_one()) {
                if (!mbar_wait(R.empty(slot), par, A.err, kErrWaitEmpty)) ok = false;
                break;
              }
            }
            if (!ok) break;
          }
          mbar_arrive_expect_tx(R.full(slot), kBlockBytes);
          bulk_g2s(smem_u32(R.base + slot * kBlockBytes), sg.base + i * (int64_t)kBlockBytes, kBlockBytes,
                   R.full(slot), pol);
          ++issued;
          if (++slot == R.nst) {
            slot = 0;
            ++round;
          }
        }
        stamp(A, cta, sgi == 4 * A.L ? 1 + 5 * A.L : 1 + 5 * (sgi >> 2) + kOpOfKind[sgi & 3], 3, 0);
      }
      flags[0] = issued;
    }
  } else if (MMA && warp == kConsumerWarps + 1) {
    // ------------------------------------------------------------ MMA issuer: every projection's blocks, in op order
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(16);
      const uint32_t zero = smem_u32(smem + Ly.zero), xop_s = smem_u32(xop);
      // Descriptors are built once: ring slot s is da0 advanced by 16 KiB x s, atom x is db0 advanced by
      // 1 KiB x x with its stride byte offset (the distance to the zero atom) shrunk by the same, and a
      // K step advances both start addresses by 32 bytes (start and offsets in 16-byte units, no carry
      // out of either 14-bit field for shared addresses below 256 KiB).
      const uint64_t da0 = umma_desc_sw128(smem_u32(R.base));
      const uint64_t db0 = umma_desc_sw128(xop_s, 16, zero - xop_s);
      const int64_t ks[K_KINDS] = {A.H, (int64_t)A.nq * 128, A.H, A.I, A.H};
      int slot = 0, fph = 0, buf = 0, xph = 0, uses[2] = {0, 0};
      bool ok = true;
      for (int sgi = 0; sgi < 4 * A.L + 1; ++sgi) {
        const int kind = (sgi == 4 * A.L) ? (int)K_LM : (sgi & 3);
        const int kblocks = (int)(ks[kind] / kBlockCols);
        const int64_t b0 = part_begin(A.total[kind], G, cta), nblk = part_begin(A.total[kind], G, cta + 1) - b0;
        if (ok) ok = mbar_wait_abort(xready, xph, A.err, kErrWaitFull, A.abort_flag);  // operand staged
        xph ^= 1;
        tc_fence_after();
        const int kb_first = (int)(b0 % kblocks);
        int kb = kb_first, sblk = 0;  // sblk: block index inside the current segment
        for (int64_t i = 0; i < nblk; ++i) {
          const bool seg_start = (i == 0) || (kb == 0);
          if (seg_start) sblk = 0;
          const bool seg_end = (kb == kblocks - 1) || (i == nblk - 1);
          if (seg_start && uses[buf] > 0 && ok)
            ok = mbar_wait_abort(acce0 + 8u * buf, (uses[buf] - 1) & 1, A.err, kErrWaitFull, A.abort_flag);
          if (ok) ok = mbar_wait_abort(R.full(slot), fph, A.err, kErrWaitFull, A.abort_flag);
          tc_fence_after();
          if (ok) {
            int sx = kb - kb_first;
            if (sx < 0) sx += kblocks;
            const uint64_t da = da0 + ((uint64_t)slot << 10);
            const uint64_t db = db0 + ((uint64_t)sx << 6) - ((uint64_t)sx << 38);
            // K = 64 per block, 16 per MMA: +32 bytes along the swizzled rows; operand rows 8..15 (the second
            // 8-row atom, at the stride byte offset) are the zero atom. The segment's k-steps go round-robin
            // to A.chains accumulators, so consecutive MMAs do not wait for one another's result; each
            // chain's first k-step of the segment overwrites it.
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int step = 4 * sblk + j, c = step & (A.chains - 1);
              umma_bf16(tmem + 16u * (buf * A.chains + c), da + 2u * j, db + 2u * j, idesc, step < A.chains ? 0u : 1u);
            }
          }
          ++sblk;
          umma_commit(R.empty(slot));  // the slot is free once these MMAs have read it
          if (seg_end) {
            umma_commit(accf0 + 8u * buf);
            ++uses[buf];
            buf ^= 1;
          }
          if (++slot == R.nst) {
            slot = 0;
            fph ^= 1;
          }
          if (++kb == kblocks) kb = 0;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    grid_dep_wait();
    int slot = 0, phase = 0;
    int abuf = 0, aph[2] = {0, 0};  // MMA variant: accumulator in use and its phases
    bool ok = true;
    // the decode position does not change during the step: read it and its RoPE rows once
    const int64_t pos = ld_cg_s64(A.pos);
    const bool pos_in = pos >= 0 && pos < A.cap;
    if (tid < 128 && pos_in) {
      aux[tid] = bf16_to_f(A.cos[pos * 128 + tid]);
      aux[128 + tid] = bf16_to_f(A.sin[pos * 128 + tid]);
    }
    if (tid == 0) {
      flags[2] = pos_in ? (int)pos : -1;
      if (!pos_in && cta == 0) atomicOr(A.err, QD_DEVERR_POS);
    }
    named_bar(kBarConsumers, kConsumers);
    // embedding: CTA i < M gathers row i (tied, packed E)
    if (cta < M) {
      int64_t t = ld_cg_s64(A.tok + cta);
      if (t < 0 || t >= A.vocab) {
        if (tid == 0) atomicOr(A.err, QD_DEVERR_TOKEN);
        t = t < 0 ? 0 : A.vocab - 1;
      }
      const int kb = A.H / kBlockCols;
      for (int q8 = tid; q8 < A.H / 8; q8 += kConsumers) {
        const uint4 v = *reinterpret_cast<const uint4*>(
            reinterpret_cast<const __nv_bfloat16*>(A.e) + packed_offset_elems(t, (int64_t)q8 * 8, kb));
        *reinterpret_cast<uint4*>(A.x + (int64_t)cta * A.H + q8 * 8) = v;
      }
      signal_done(A.counters, tid);
    }
    stamp(A, cta, 0, 2, tid);
    const int team = warp >> 2, team_tid = tid & (kAttnThreads - 1);
    const int units = M * A.nkv * A.splits;
    const int64_t len = attn_len_of(A, pos);
    int64_t achunk;
    const int n_use = attn_active_of(A, len, &achunk);
    // short caches: attention folded into the QKV epilogue (the same for every CTA: one position per step)
    const bool fold = len <= A.fold_max;
    if (tid == 0) flags[4] = 0;
    for (int l = 0; l < A.L; ++l) {
      // Off the critical path, at the start of the layer: prefetch into L2 what this layer reads that
      // does not depend on this step's activations - the cached keys / values of this CTA's attention
      // units (every position but the new one) and the layer's small RMSNorm weights (the weight
      // stream, with its evict-first policy, keeps them out of L2 otherwise).
      {
        const int per_b = A.nkv * A.splits;
        if (fold) {  // the folding CTAs are known only later: CTA c prefetches keys c, c + G, ... of all heads
          for (int t = cta * kConsumers + tid; t < M * A.nkv * (len - 1); t += G * kConsumers) {
            const int64_t key = t % (len - 1), bh = t / (len - 1);
            const int64_t off = l * A.c_ls + (bh / A.nkv) * A.cs_b + (bh % A.nkv) * A.cs_h + key * kHeadDim;
            prefetch_l2(A.kc + off, kHeadDim * 2);
            prefetch_l2(A.vc + off, kHeadDim * 2);
          }
        }
        for (int u = fold ? units : cta + team * G; u < units; u += 2 * G) {
          const int b = u / per_b, rem = u - b * per_b, kvh = rem / A.splits, sp = rem % A.splits;
          if (sp >= n_use) continue;
          const int64_t k0 = sp * achunk, k1 = (k0 + achunk < len - 1) ? k0 + achunk : len - 1;
          const int64_t off = l * A.c_ls + b * A.cs_b + kvh * A.cs_h;
          for (int64_t kk = k0 + team_tid * 32; kk < k1; kk += kAttnThreads * 32) {
            const uint32_t bytes = (uint32_t)((k1 - kk < 32 ? k1 - kk : 32) * kHeadDim * 2);
            prefetch_l2(A.kc + off + kk * kHeadDim, bytes);
            prefetch_l2(A.vc + off + kk * kHeadDim, bytes);
          }
        }
        const int hb = A.H * 2;  // bytes of one norm weight row (multiple of 256)
        if (tid == 0) {
          prefetch_l2(A.ln1 + (int64_t)l * A.H, hb);
          prefetch_l2(A.ln2 + (int64_t)l * A.H, hb);
          prefetch_l2(A.qn + (int64_t)l * 128, 256);
          prefetch_l2(A.kn + (int64_t)l * 128, 256);
          if (l == A.L - 1) prefetch_l2(A.fnorm, hb);
        }
      }
      // QKV projection + q/k norm + RoPE + K/V append
      wait_dep(A, l == 0 ? A.counters : ctr(A, l - 1, 4), l == 0 ? M : A.H / kBlockRows, tid);
      stamp(A, cta, 1 + 5 * l, 0, tid);
      {
        GemvArgs op = gemv_op<M>(A, K_QKV, l);
        if (fold) op.finalized = flags + 4;  // the row groups this CTA finalizes, for the folded attention
        step_stage<M, MMA>(op, cta, xs, xop, xready, wsum, tid);
        stamp(A, cta, 1 + 5 * l, 1, tid);
        step_consume<M, MODE_QKV, MMA>(op, R, slot, phase, cta, xs, tmem, A.chains, accf0, acce0, abuf, aph, red, wsum,
                                             lmv, lmi, flags, aux, A.abort_flag, tid, ok);
        if (fold) fold_after_qkv<M>(A, cta, l, len, flags + 4, flags, *reinterpret_cast<FoldSmem*>(asm_team), tid);
      }
      stamp(A, cta, 1 + 5 * l, 2, tid);
      // attention: units (sequence, KV head, split) over CTAs, two teams of 4 warps per CTA. The cached
      // keys / values (all but the new one the QKV epilogue appends) do not depend on this layer's
      // projection, so each unit's range is prefetched into L2 before waiting for it.
      {
        AttnArgs at = {};
        at.q = A.q;
        at.k = A.kc + l * A.c_ls;
        at.v = A.vc + l * A.c_ls;
        at.pos = A.pos;
        at.out = A.attn;
        at.batch = M;
        at.nq = A.nq;
        at.nkv = A.nkv;
        at.splits = A.splits;
        at.cap = A.cap;
        at.cs_b = A.cs_b;
        at.cs_h = A.cs_h;
        at.chunk = A.chunk;
        at.scale = A.scale;
        at.part_acc = A.attn_acc;
        at.part_ml = A.attn_ml;
        at.tickets = A.attn_tickets;
        at.err = A.err;
        at.done = ctr(A, l, 1);
        at.keys_per_split = A.keys_per_split;
        at.partials_only = A.o_merge;
        const int per_b = A.nkv * A.splits;
        if (!fold) {
          wait_dep(A, ctr(A, l, 0), A.nq + 2 * A.nkv, tid);
          stamp(A, cta, 2 + 5 * l, 0, tid);
          for (int u = cta + team * G; u < units; u += 2 * G) {
            const int b = u / per_b, rem = u - b * per_b;
            attn_unit(at, b, rem / A.splits, rem % A.splits, team_tid, 2 + team, asm_team[team], len);
          }
        }
      }
      stamp(A, cta, 2 + 5 * l, 2, tid);
      // O projection + residual
      wait_dep(A, ctr(A, l, 1), fold ? A.nkv : (A.o_merge ? M * A.nkv * n_use : M * A.nkv), tid);
      stamp(A, cta, 3 + 5 * l, 0, tid);
      {
        const GemvArgs op = gemv_op<M>(A, K_O, l);
        if (A.o_merge && !fold) {
          stage_attn_merge<M, MMA>(A, op, n_use, cta, xs, xop, reinterpret_cast<float*>(asm_team), tid);
          if (MMA && tid == 0) mbar_arrive(xready);
        } else {
          step_stage<M, MMA>(op, cta, xs, xop, xready, wsum, tid);
        }
        stamp(A, cta, 3 + 5 * l, 1, tid);
        step_consume<M, MODE_RES, MMA>(op, R, slot, phase, cta, xs, tmem, A.chains, accf0, acce0, abuf, aph, red, wsum,
                                             lmv, lmi, flags, aux, A.abort_flag, tid, ok);
      }
      stamp(A, cta, 3 + 5 * l, 2, tid);
      // gate_up + SwiGLU
      wait_dep(A, ctr(A, l, 2), A.H / kBlockRows, tid);
      stamp(A, cta, 4 + 5 * l, 0, tid);
      {
        const GemvArgs op = gemv_op<M>(A, K_GU, l);
        step_stage<M, MMA>(op, cta, xs, xop, xready, wsum, tid);
        stamp(A, cta, 4 + 5 * l, 1, tid);
        step_consume<M, MODE_SWIGLU, MMA>(op, R, slot, phase, cta, xs, tmem, A.chains, accf0, acce0, abuf, aph, red, wsum,
                                             lmv, lmi, flags, aux, A.abort_flag, tid, ok);
      }
      stamp(A, cta, 4 + 5 * l, 2, tid);
      // down projection + residual
      wait_dep(A, ctr(A, l, 3), 2 * A.I / kBlockRows, tid);
      stamp(A, cta, 5 + 5 * l, 0, tid);
      {
        const GemvArgs op = gemv_op<M>(A, K_DOWN, l);
        step_stage<M, MMA>(op, cta, xs, xop, xready, wsum, tid);
        stamp(A, cta, 5 + 5 * l, 1, tid);
        step_consume<M, MODE_RES, MMA>(op, R, slot, phase, cta, xs, tmem, A.chains, accf0, acce0, abuf, aph, red, wsum,
                                             lmv, lmi, flags, aux, A.abort_flag, tid, ok);
      }
      stamp(A, cta, 5 + 5 * l, 2, tid);
    }
    // LM head + argmax + position advance; the last CTA also clears the counters for the next step
    wait_dep(A, ctr(A, A.L - 1, 4), A.H / kBlockRows, tid);
    stamp(A, cta, 1 + 5 * A.L, 0, tid);
    {
      const GemvArgs op = gemv_op<M>(A, K_LM, 0);
      step_stage<M, MMA>(op, cta, xs, xop, xready, wsum, tid);
      stamp(A, cta, 1 + 5 * A.L, 1, tid);
      step_consume<M, MODE_LM, MMA>(op, R, slot, phase, cta, xs, tmem, A.chains, accf0, acce0, abuf, aph, red, wsum,
                                             lmv, lmi, flags, aux, A.abort_flag, tid, ok);
      stamp(A, cta, 1 + 5 * A.L, 2, tid);
      if (lm_global_argmax<M>(op, cta, wsum, lmv, lmi, flags, tid)) {
        for (int i = tid; i < 1 + 5 * A.L; i += kConsumers) A.counters[i] = 0;
      }
    }
  }
  if constexpr (MMA) tc_fence_before();
  __syncthreads();
  if constexpr (MMA) {
    tc_fence_after();
    if (warp == kConsumerWarps + 1) tmem_dealloc(tmem, 256);
  }
  if (tid == 0) ring_drain(R, flags[0], A.err);
}

struct StepPlan {
  int grid, nst, splits, kmax, smem, o_merge, mma, xatoms;
  int64_t chunk;
  int smax[K_KINDS];
  int64_t total[K_KINDS];
  int64_t off_counters, off_abort, off_tickets, off_lm_ticket, off_cta_val, off_cta_idx, off_partials, off_attn_acc,
      off_attn_ml, off_attn_tickets, off_kv_tickets, bytes;
};

static int step_plan(const qd_step_desc* d, StepPlan* p) {
  if (!d) return set_error(QD_ERR_ARG, "null step descriptor");
  const int64_t L = d->layers, H = d->hidden, I = d->inter, nq = d->nq_heads, nkv = d->nkv_heads, B = d->batch;
  if (L < 1 || H < 64 || H % 128 || I % 64 || (2 * I) % 128 || nq != 4 * nkv || nkv < 1 || (nq * 128) % 64 ||
      d->vocab < 1 || B < 1 || B > 8 || d->cap < 1)
    return set_error(QD_ERR_UNSUPPORTED, "step: unsupported shape (H %% 128, I %% 64, 4 q heads per KV head, "
                                         "head_dim 128, 1 <= batch <= 8)");
  const int G = host_sm_count();
  p->grid = G;
  const int64_t vocab_rows = (d->vocab + kBlockRows - 1) / kBlockRows * kBlockRows;
  const int64_t n_rows[K_KINDS] = {(nq + 2 * nkv) * 128, H, 2 * I, H, vocab_rows};
  const int64_t ks[K_KINDS] = {H, nq * 128, H, I, H};
  int64_t max_groups = 0, max_partials = 0;
  for (int k = 0; k < K_KINDS; ++k) {
    const int64_t groups = n_rows[k] / kBlockRows;
    const int kblocks = (int)(ks[k] / kBlockCols);
    p->total[k] = groups * kblocks;
    if (p->total[k] < G) return set_error(QD_ERR_UNSUPPORTED, "step: a projection has fewer blocks than SMs");
    p->smax[k] = stream_k_smax(groups, kblocks, G);
    if (groups > max_groups) max_groups = groups;
    const int64_t part = groups * p->smax[k] * B * kBlockRows * 4;
    if (part > max_partials) max_partials = part;
  }
  AttnPlan ap;
  if (!attn_plan((int)B, (int)nkv, d->cap, 2 * G, &ap)) return set_error(QD_ERR_ARG, "step: attention plan");
  p->splits = ap.splits;
  p->chunk = ap.chunk;
  int64_t kmax = H;
  if (nq * 128 > kmax) kmax = nq * 128;
  if (I > kmax) kmax = I;
  p->kmax = (int)kmax;
  // QD_STEP_MMA (default 0): 1 = the tensor-core consumers, 0 = the CUDA-core consumers. The tensor-core B
  // operand holds the k-blocks one CTA's range of a projection touches: at most min(k / 64, range).
  p->mma = env_int("QD_STEP_MMA", 0) != 0 ? 1 : 0;
  p->xatoms = 0;
  for (int k = 0; k < K_KINDS; ++k) {
    const int64_t kb = ks[k] / kBlockCols, range = (p->total[k] + G - 1) / G;
    const int need = (int)(range < kb ? range : kb);
    if (need > p->xatoms) p->xatoms = need;
  }
  const int fixed = p->mma ? step_mma_layout((int)B, p->xatoms, 0).total + 1024 : step_layout((int)B, p->kmax, 0).total;
  int nst = (227 * 1024 - fixed) / (kBlockBytes + (p->mma ? 16 + 8 : 16));
  const int cap_st = env_int("QD_STEP_STAGES", 16);  // tuning: upper bound on the ring depth
  if (nst > cap_st) nst = cap_st;
  if (nst > 16) nst = 16;
  if (nst < 2) return set_error(QD_ERR_UNSUPPORTED, "step: shared memory too small for batch %lld", (long long)B);
  auto smem_of = [&](int n) {
    return p->mma ? step_mma_layout((int)B, p->xatoms, n).total + 1024 : step_layout((int)B, p->kmax, n).total;
  };
  while (nst > 2 && smem_of(nst) > 227 * 1024) --nst;
  p->nst = nst;
  p->smem = smem_of(nst);
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  p->off_counters = take((1 + 5 * L) * 4);
  p->off_abort = take(4);
  p->off_tickets = take(max_groups * 4);
  p->off_lm_ticket = take(4);
  p->off_cta_val = take(B * G * 4);
  p->off_cta_idx = take(B * G * 4);
  p->off_partials = take(max_partials);
  p->off_attn_acc = take(B * nq * ap.splits * 128 * 4);
  p->off_attn_ml = take(B * nq * ap.splits * 2 * 4);
  p->off_attn_tickets = take(B * nkv * 4);
  p->off_kv_tickets = take(nkv * 4);
  p->bytes = off;
  // O-side attention merge: the most query heads one O CTA reads, times the splits, must fit the
  // attention shared memory (free while O stages its input); heads as bits of a 32-bit mask
  {
    const int64_t T = p->total[K_O], kbl = nq * 128 / kBlockCols;
    int nh_max = 0;
    for (int c = 0; c < G; ++c) {
      uint32_t mask = 0;
      for (int64_t b = part_begin(T, G, c); b < part_begin(T, G, c + 1); ++b) mask |= 1u << ((b % kbl) >> 1);
      const int nh = __builtin_popcount(mask);
      if (nh > nh_max) nh_max = nh;
    }
    const int64_t need = (3 * (int64_t)ap.splits + 1) * B * nh_max;
    const int64_t cap_f = 2 * (int64_t)sizeof(AttnSmem) / 4;
    p->o_merge = (nq <= 32 && need <= cap_f && env_int("QD_STEP_O_MERGE", 1) != 0) ? 1 : 0;
  }
  return QD_OK;
}

template <int M, bool MMA>
static int launch_step(const StepArgs& a, int smem, cudaStream_t stream) {
  auto kern = step_kernel<M, MMA>;
  const int threads = MMA ? kThreads + 32 : kThreads;
  if (int rc = set_max_dynamic_smem((const void*)kern, smem)) return rc;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  if (e != cudaSuccess || per_sm < 1)
    return set_error(QD_ERR_UNSUPPORTED, "step kernel does not fit on an SM (smem %d B)", smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: CTAs wait on one another's results
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[1] = {(void*)&a};
  e = cudaLaunchKernelExC(&cfg, (const void*)kern, args);
  if (e != cudaSuccess) return set_error(QD_ERR_CUDA, "step launch: %s", cudaGetErrorString(e));
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(QD_ERR_CUDA, "step launch: %s", cudaGetErrorString(e));
  return QD_OK;
}

}  // namespace qd

using namespace qd;

extern "C" int qd_decode_step_plan(const qd_step_desc* d, int64_t* scratch_bytes, int* attn_splits) {
  StepPlan p;
  if (int rc = step_plan(d, &p)) return rc;
  if (scratch_bytes) *scratch_bytes = p.bytes;
  if (attn_splits) *attn_splits = p.splits;
  return QD_OK;
}

extern "C" int qd_decode_step(const qd_step_desc* d, void* scratch, int64_t scratch_bytes, cudaStream_t stream) {
  StepPlan p;
  if (int rc = step_plan(d, &p)) return rc;
  if (!scratch || scratch_bytes < p.bytes)
    return set_error(QD_ERR_SCRATCH, "scratch %lld B < %lld B", (long long)scratch_bytes, (long long)p.bytes);
  const void* ptrs[] = {d->w_qkv, d->w_o, d->w_gu, d->w_down, d->e_packed, d->ln1, d->ln2, d->q_norm, d->k_norm,
                        d->final_norm, d->tok, d->pos, d->x, d->q, d->attn, d->act, d->k_cache, d->v_cache, d->cos,
                        d->sin, d->err};
  for (const void* q : ptrs)
    if (!q) return set_error(QD_ERR_ARG, "step: null pointer in the descriptor");
  for (const void* q : {d->w_qkv, d->w_o, d->w_gu, d->w_down, d->e_packed, (const void*)d->x, (const void*)d->q,
                        (const void*)d->attn, (const void*)d->act, (const void*)d->k_cache, (const void*)d->v_cache,
                        d->ln1, d->ln2, d->final_norm})
    if (!aligned16(q)) return set_error(QD_ERR_ARG, "step: buffers must be 16-byte aligned");
  if (d->cs_h < d->cap * 128 || d->cs_b < d->nkv_heads * d->cs_h || d->cache_layer_stride < d->batch * d->cs_b ||
      d->cs_h % 8 || d->cs_b % 8 || d->cache_layer_stride % 8)
    return set_error(QD_ERR_ARG, "step: cache strides");
  if (d->logits && d->ld_logits < d->vocab) return set_error(QD_ERR_ARG, "step: ld_logits < vocab");
  const int64_t H = d->hidden, I = d->inter, nq = d->nq_heads, nkv = d->nkv_heads;
  const int64_t need_qkv = (nq + 2 * nkv) * 128 * H * 2, need_o = H * nq * 128 * 2, need_gu = 2 * I * H * 2,
                need_down = H * I * 2;
  if (d->w_qkv_layer_bytes < need_qkv || d->w_o_layer_bytes < need_o || d->w_gu_layer_bytes < need_gu ||
      d->w_down_layer_bytes < need_down)
    return set_error(QD_ERR_ARG, "step: per-layer weight strides smaller than the packed matrices");
  StepArgs a = {};
  a.w_qkv = static_cast<const char*>(d->w_qkv);
  a.w_o = static_cast<const char*>(d->w_o);
  a.w_gu = static_cast<const char*>(d->w_gu);
  a.w_down = static_cast<const char*>(d->w_down);
  a.e = static_cast<const char*>(d->e_packed);
  a.qkv_lb = d->w_qkv_layer_bytes;
  a.o_lb = d->w_o_layer_bytes;
  a.gu_lb = d->w_gu_layer_bytes;
  a.down_lb = d->w_down_layer_bytes;
  a.ln1 = static_cast<const __nv_bfloat16*>(d->ln1);
  a.ln2 = static_cast<const __nv_bfloat16*>(d->ln2);
  a.qn = static_cast<const __nv_bfloat16*>(d->q_norm);
  a.kn = static_cast<const __nv_bfloat16*>(d->k_norm);
  a.fnorm = static_cast<const __nv_bfloat16*>(d->final_norm);
  a.L = (int)d->layers;
  a.H = (int)H;
  a.I = (int)I;
  a.nq = (int)nq;
  a.nkv = (int)nkv;
  a.vocab = d->vocab;
  a.vocab_rows = (d->vocab + kBlockRows - 1) / kBlockRows * kBlockRows;
  a.eps = (float)d->eps;
  a.o_merge = p.o_merge;
  a.scale = (float)d->scale;
  a.tok = d->tok;
  a.pos = d->pos;
  a.x = static_cast<__nv_bfloat16*>(d->x);
  a.q = static_cast<__nv_bfloat16*>(d->q);
  a.attn = static_cast<__nv_bfloat16*>(d->attn);
  a.act = static_cast<__nv_bfloat16*>(d->act);
  a.kc = static_cast<__nv_bfloat16*>(d->k_cache);
  a.vc = static_cast<__nv_bfloat16*>(d->v_cache);
  a.c_ls = d->cache_layer_stride;
  a.cs_b = d->cs_b;
  a.cs_h = d->cs_h;
  a.cap = d->cap;
  a.cos = static_cast<const __nv_bfloat16*>(d->cos);
  a.sin = static_cast<const __nv_bfloat16*>(d->sin);
  a.logits = static_cast<__nv_bfloat16*>(d->logits);
  a.ld_logits = d->ld_logits;
  a.err = d->err;
  a.grid = p.grid;
  a.nst = p.nst;
  a.prefetch = prefetch_blocks();
  a.prefetch_max = env_int("QD_PREFETCH_MAX_BLOCKS", 8);
  if (a.prefetch_max < a.prefetch) a.prefetch_max = a.prefetch;
  a.evict_first = env_int("QD_EVICT_FIRST", 1) != 0;
  a.keys_per_split = attn_keys_per_split();
  a.splits = p.splits;
  a.kmax = p.kmax;
  a.chunk = p.chunk;
  for (int k = 0; k < K_KINDS; ++k) {
    a.smax[k] = p.smax[k];
    a.total[k] = p.total[k];
  }
  char* sc = static_cast<char*>(scratch);
  a.counters = reinterpret_cast<int*>(sc + p.off_counters);
  a.abort_flag = reinterpret_cast<int*>(sc + p.off_abort);
  a.tickets = reinterpret_cast<int*>(sc + p.off_tickets);
  a.lm_ticket = reinterpret_cast<int*>(sc + p.off_lm_ticket);
  a.trace = d->trace;
  a.cta_val = reinterpret_cast<float*>(sc + p.off_cta_val);
  a.cta_idx = reinterpret_cast<int*>(sc + p.off_cta_idx);
  a.partials = reinterpret_cast<float*>(sc + p.off_partials);
  a.attn_acc = reinterpret_cast<float*>(sc + p.off_attn_acc);
  a.attn_ml = reinterpret_cast<float*>(sc + p.off_attn_ml);
  a.attn_tickets = reinterpret_cast<int*>(sc + p.off_attn_tickets);
  a.kv_tickets = reinterpret_cast<int*>(sc + p.off_kv_tickets);
  // QD_STEP_ATTN_FOLD: longest valid length (keys) whose attention is folded into the QKV epilogue
  a.fold_max = env_int("QD_STEP_ATTN_FOLD", 0);
  a.xatoms = p.xatoms;
  {  // QD_STEP_MMA_CHAINS: accumulators a segment's MMAs rotate over (1, 2, 4 or 8; default 8)
    const int c = env_int("QD_STEP_MMA_CHAINS", 8);
    a.chains = c >= 8 ? 8 : (c >= 4 ? 4 : (c >= 2 ? 2 : 1));
  }
  switch (d->batch * 2 + p.mma) {
    case 2: return launch_step<1, false>(a, p.smem, stream);
    case 3: return launch_step<1, true>(a, p.smem, stream);
    case 4: return launch_step<2, false>(a, p.smem, stream);
    case 5: return launch_step<2, true>(a, p.smem, stream);
    case 6: return launch_step<3, false>(a, p.smem, stream);
    case 7: return launch_step<3, true>(a, p.smem, stream);
    case 8: return launch_step<4, false>(a, p.smem, stream);
    case 9: return launch_step<4, true>(a, p.smem, stream);
    case 10: return launch_step<5, false>(a, p.smem, stream);
    case 11: return launch_step<5, true>(a, p.smem, stream);
    case 12: return launch_step<6, false>(a, p.smem, stream);
    case 13: return launch_step<6, true>(a, p.smem, stream);
    case 14: return launch_step<7, false>(a, p.smem, stream);
    case 15: return launch_step<7, true>(a, p.smem, stream);
    case 16: return launch_step<8, false>(a, p.smem, stream);
    case 17: return launch_step<8, true>(a, p.smem, stream);
  }
  return set_error(QD_ERR_UNSUPPORTED, "batch %lld", (long long)d->batch);
}
