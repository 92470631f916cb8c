// Persistent whole-decode-step kernel, sm_100a: one launch runs embedding -> layers x [QKV + q/k
// norm + RoPE + KV append, attention, O + residual, gate_up + SwiGLU, down + residual] -> LM head +
// argmax + position advance.
//
// One CTA per SM (cooperative launch, so every CTA is resident). The producer warp streams this
// CTA's share of every projection's weight blocks, op after op and layer after layer, into one deep
// ring of 16 KiB blocks: weights never depend on activations, so HBM keeps streaming the next
// projection while the consumers wait for the current one's inputs. The eight consumer warps walk
// the same op sequence; before each op, one thread waits (bounded) on the completion counter of the
// op that produces its input, e.g. down waits until all row groups of gate_up are finalized. Counters
// are bumped with release semantics by whoever finalizes a row group (a GEMV epilogue) or merges a
// (sequence, KV head) (attention); all cross-CTA activations are read with L2 (.cg) loads after an
// acquire. The residual projections (O, down) finalize nothing: every CTA adds its partial sums into
// fixed-point group sums with integer atomics and its K-block count into the op's counter, and the next
// op's staging (gate/up, the next layer's QKV, the LM head) applies the residual add itself once the
// count is complete - no last-arriving CTA's reduction sits between the two ops. The per-op arithmetic
// is the per-projection kernels' (qd_gemv_dev.cuh, qd_attn_dev.cuh; their residual projections sum
// their partials in the same fixed point) with the same stream-K partition and attention splits, so
// the two paths produce bit-identical tokens and logits.
//
// Failure handling: every wait is bounded (1 s); a dependency wait that expires sets QD_DEVERR_DEP
// and an abort flag that makes every later wait return at once, so a broken step finishes (with
// garbage) instead of hanging. The host reads the error word and clears the scratch.
#include "qd_attn_dev.cuh"
#include "qd_gemv_dev.cuh"
#include "qd_plan.h"

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
  int64_t chunk;
  int smax[K_KINDS];
  int64_t total[K_KINDS];
  int o_merge;       // 1: attention leaves split partials, the O projection's CTAs merge them
  // The O and down projections leave their outputs as fixed-point group sums (fx_o, fx_d: [M][H] int64)
  // and the next op's staging applies the residual add; the residual stream alternates between x (a
  // layer's input) and xb (after its O projection)
  __nv_bfloat16* xb;
  int64_t *fx_o, *fx_d;
  // The QKV projection likewise leaves fixed-point sums (fx_q: [M][(nq + 2 nkv) * 128]); each attention
  // unit applies the QKV epilogue (per-head RMSNorm, RoPE) to its own query heads, and the unit that
  // covers the new position also to the new key / value, which it appends to the cache
  int64_t* fx_q;
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
  off += 16;
  L.aux = off;
  off += 512 * 4;
  L.attn = sal(off, 16);
  static_assert(sizeof(AttnSmem) % 16 == 0, "attention team buffers must stay 16-byte aligned");
  off = L.attn + 2 * (int)sizeof(AttnSmem);
  L.bars = sal(off, 8);
  off = L.bars + 2 * nst * 8;
  L.total = sal(off, 128);
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
  if (tid == 0) wait_count_ge(cnt, target, A.abort_flag, A.err, kErrDep);
  named_bar(kBarConsumers, kConsumers);
}

// The O projection's input at batch 1..8: attention units leave their split partials (acc, max, sum)
// and each O CTA merges, for the query heads its K-range reads (K-block kb = dims 64kb.. = head kb/2),
// exactly what the attention kernel's last split computes (same order, same operations), into xs.
// Saves the split ticket, the merge's round trips and the output write + reload on the critical path.
template <int M>
static __device__ void stage_attn_merge(const StepArgs& A, const GemvArgs& op, int n_use, int cta,
                                        __nv_bfloat16* xs, float* scr, int tid) {
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
    xs[(int64_t)m * op.k + hq * kHeadDim + d] = __float2bfloat16_rn(num / den[p]);
  }
  named_bar(kBarConsumers, kConsumers);
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
    a.x = l > 0 ? A.xb : A.x;  // the residual stream before the previous layer's down projection
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
    a.pos_ready = 1;
    a.fx_numerics = 1;
    a.fx = A.fx_q;
    a.fx_ctr = ctr(A, l, 0);
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
    a.fx_numerics = 1;
    a.fx = A.fx_o;
    a.fx_ctr = ctr(A, l, 2);
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
    a.fx_numerics = 1;
    a.fx = A.fx_d;
    a.fx_ctr = ctr(A, l, 4);
  } else {  // LM head
    a.x = A.xb;
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

// The QKV epilogue of one attention unit from the fixed-point QKV sums - the arithmetic of
// finalize_group's QKV mode: BF16 projection output, per-head RMSNorm (sum of squares per 32 rows, the 4
// slices added in order), q_norm / k_norm, RoPE at position p with every product rounded to BF16. The
// unit's 4 query heads go to sm.qs (BF16 values as floats); with `append` (the unit whose keys include
// the new position) the new key and value of KV head kvh are written to the cache at p. A team of 128
// threads, one per dimension r; named barrier bar_id. cs: cos[0..127], sin[128..255] at p.
static __device__ void qkv_heads_from_sums(const StepArgs& A, int l, int b, int kvh, bool append, int64_t p,
                                           const float* cs, int r, int bar_id, AttnSmem& sm) {
  const int64_t nqkv = (int64_t)(A.nq + 2 * A.nkv) * 128;
  const int64_t* row = A.fx_q + (int64_t)b * nqkv;
  const int lane = r & 31, w = r >> 5;
  const int nh = append ? kGroup + 1 : kGroup;  // 4 query heads, then the key head
  float* ys = &sm.wacc[0][0][0];                 // [5][128] normalised values (partner exchange)
  float* wsq = ys + (kGroup + 1) * kHeadDim;     // [5][4] per-slice sums of squares
  float v[kGroup + 1];
  for (int hh = 0; hh < nh; ++hh) {
    const int g = hh < kGroup ? kvh * kGroup + hh : A.nq + kvh;
    v[hh] = bf16r(fx_to_float(__ldcg(row + (int64_t)g * kHeadDim + r)));
  }
  const float vv = append ? bf16r(fx_to_float(__ldcg(row + (int64_t)(A.nq + A.nkv + kvh) * kHeadDim + r))) : 0.f;
  const float nwq = bf16_to_f(A.qn[(int64_t)l * kHeadDim + r]), nwk = bf16_to_f(A.kn[(int64_t)l * kHeadDim + r]);
  for (int hh = 0; hh < nh; ++hh) {
    const float sq = warp_sum(v[hh] * v[hh]);
    if (lane == 0) wsq[hh * 4 + w] = sq;
  }
  named_bar(bar_id, kAttnThreads);
  for (int hh = 0; hh < nh; ++hh) {
    const float var = (wsq[hh * 4 + 0] + wsq[hh * 4 + 1] + wsq[hh * 4 + 2] + wsq[hh * 4 + 3]) / 128.0f;
    const float rstd = 1.0f / sqrtf(var + A.eps);
    ys[hh * kHeadDim + r] = bf16r((hh < kGroup ? nwq : nwk) * bf16r(v[hh] * rstd));
  }
  named_bar(bar_id, kAttnThreads);
  const float c = cs[r], sn = cs[128 + r];
  for (int hh = 0; hh < nh; ++hh) {
    const float y = ys[hh * kHeadDim + r], yp = ys[hh * kHeadDim + (r ^ 64)];
    // q*cos + rotate_half(q)*sin with every product a BF16 tensor (rotate_half = cat(-q2, q1))
    const float rot = (r < 64) ? bf16r(-yp * sn) : bf16r(yp * sn);
    const __nv_bfloat16 o = __float2bfloat16_rn(bf16r(y * c) + rot);
    if (hh < kGroup) {
      sm.qs[hh][r] = __bfloat162float(o);
    } else if (p >= 0) {
      const int64_t off = (int64_t)l * A.c_ls + (int64_t)b * A.cs_b + (int64_t)kvh * A.cs_h + p * kHeadDim + r;
      A.kc[off] = o;
      A.vc[off] = __float2bfloat16_rn(vv);
    }
  }
  named_bar(bar_id, kAttnThreads);  // queries complete, the new key / value written, before the unit reads
}

template <int M>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const __grid_constant__ StepArgs A) {
  extern __shared__ __align__(1024) char smem[];
  const StepLayout Ly = step_layout(M, A.kmax, A.nst);
  const Ring R{smem + Ly.ring, smem_u32(smem + Ly.bars), A.nst};
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + Ly.xs);
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
    ring_init(R);
    flags[0] = 0;
    flags[1] = 0;
  }
  if (tid < M) {
    lmv[tid] = -INFINITY;
    lmi[tid] = 0x7fffffff;
  }
  __syncthreads();

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
  } else {
    // ------------------------------------------------------------ consumers
    grid_dep_wait();
    int slot = 0, phase = 0;
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
    // this CTA's share of a [M][H] fixed-point sum buffer, cleared with plain stores (the CTA's later
    // releases publish them before any other CTA adds into the buffer again)
    auto zero_share = [&](int64_t* buf, int64_t row_elems) {
      const int64_t E = (int64_t)M * row_elems, e0 = E * cta / G, e1 = E * (cta + 1) / G;
      for (int64_t e = e0 + tid; e < e1; e += kConsumers) buf[e] = 0;
    };
    const int units = M * A.nkv * A.splits;
    const int64_t len = attn_len_of(A, pos);
    int64_t achunk;
    const int n_use = attn_active_of(A, len, &achunk);
    for (int l = 0; l < A.L; ++l) {
      // Off the critical path, at the start of the layer: prefetch into L2 what this layer reads that
      // does not depend on this step's activations - the cached keys / values of this CTA's attention
      // units (every position but the new one) and the layer's small RMSNorm weights (the weight
      // stream, with its evict-first policy, keeps them out of L2 otherwise).
      {
        const int per_b = A.nkv * A.splits;
        for (int u = cta + team * G; u < units; u += 2 * G) {
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
      wait_dep(A, l == 0 ? A.counters : ctr(A, l - 1, 4), l == 0 ? M : (int)A.total[K_DOWN], tid);
      stamp(A, cta, 1 + 5 * l, 0, tid);
      {
        const GemvArgs op = gemv_op<M>(A, K_QKV, l);
        if (l > 0)  // x = previous layer's (x after O) + down's sums; this CTA's share to x
          stage_x_fx<M>(op, A.fx_d, A.x, cta, G, xs, wsum, tid);
        else
          stage_x<M>(op, xs, wsum, tid);
        stamp(A, cta, 1 + 5 * l, 1, tid);
        consume_blocks<M, MODE_QKV, true>(op, R, slot, phase, cta, xs, red, wsum, lmv, lmi, flags, aux, tid, ok);
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
        wait_dep(A, ctr(A, l, 0), (int)A.total[K_QKV], tid);
        // every CTA has contributed to this layer's QKV, so all have staged the down sums they read: clear
        // this CTA's share for the next layer's down
        if (l > 0) zero_share(A.fx_d, A.H);
        stamp(A, cta, 2 + 5 * l, 0, tid);
        for (int u = cta + team * G; u < units; u += 2 * G) {
          const int b = u / per_b, rem = u - b * per_b, kvh = rem / A.splits, sp = rem % A.splits;
          if (sp >= n_use) continue;  // beyond the splits in use at this length (attn_unit would return)
          qkv_heads_from_sums(A, l, b, kvh, sp == n_use - 1, flags[2], aux, team_tid, 2 + team, asm_team[team]);
          attn_unit(at, b, kvh, sp, team_tid, 2 + team, asm_team[team], len, true);
        }
      }
      stamp(A, cta, 2 + 5 * l, 2, tid);
      // O projection + residual
      wait_dep(A, ctr(A, l, 1), A.o_merge ? M * A.nkv * n_use : M * A.nkv, tid);
      // every attention unit has read its QKV sums: clear this CTA's share for the next layer's QKV
      zero_share(A.fx_q, (int64_t)(A.nq + 2 * A.nkv) * 128);
      stamp(A, cta, 3 + 5 * l, 0, tid);
      {
        const GemvArgs op = gemv_op<M>(A, K_O, l);
        if (A.o_merge)
          stage_attn_merge<M>(A, op, n_use, cta, xs, reinterpret_cast<float*>(asm_team), tid);
        else
          stage_x<M>(op, xs, wsum, tid);
        stamp(A, cta, 3 + 5 * l, 1, tid);
        consume_blocks<M, MODE_RES, true>(op, R, slot, phase, cta, xs, red, wsum, lmv, lmi, flags, aux, tid, ok);
      }
      stamp(A, cta, 3 + 5 * l, 2, tid);
      // gate_up + SwiGLU
      wait_dep(A, ctr(A, l, 2), (int)A.total[K_O], tid);
      stamp(A, cta, 4 + 5 * l, 0, tid);
      {
        const GemvArgs op = gemv_op<M>(A, K_GU, l);
        stage_x_fx<M>(op, A.fx_o, A.xb, cta, G, xs, wsum, tid);  // x after O = x + O's sums; share to xb
        stamp(A, cta, 4 + 5 * l, 1, tid);
        consume_blocks<M, MODE_SWIGLU>(op, R, slot, phase, cta, xs, red, wsum, lmv, lmi, flags, aux, tid, ok);
      }
      stamp(A, cta, 4 + 5 * l, 2, tid);
      // down projection + residual
      wait_dep(A, ctr(A, l, 3), 2 * A.I / kBlockRows, tid);
      zero_share(A.fx_o, A.H);  // every CTA has staged gate/up, so O's sums are read: clear this CTA's share
      stamp(A, cta, 5 + 5 * l, 0, tid);
      {
        const GemvArgs op = gemv_op<M>(A, K_DOWN, l);
        stage_x<M>(op, xs, wsum, tid);
        stamp(A, cta, 5 + 5 * l, 1, tid);
        consume_blocks<M, MODE_RES, true>(op, R, slot, phase, cta, xs, red, wsum, lmv, lmi, flags, aux, tid, ok);
      }
      stamp(A, cta, 5 + 5 * l, 2, tid);
    }
    // LM head + argmax + position advance; the last CTA also clears the counters for the next step
    wait_dep(A, ctr(A, A.L - 1, 4), (int)A.total[K_DOWN], tid);
    stamp(A, cta, 1 + 5 * A.L, 0, tid);
    {
      const GemvArgs op = gemv_op<M>(A, K_LM, 0);
      stage_x_fx<M>(op, A.fx_d, nullptr, cta, G, xs, wsum, tid);
      stamp(A, cta, 1 + 5 * A.L, 1, tid);
      consume_blocks<M, MODE_LM>(op, R, slot, phase, cta, xs, red, wsum, lmv, lmi, flags, aux, tid, ok);
      stamp(A, cta, 1 + 5 * A.L, 2, tid);
      if (lm_global_argmax<M>(op, cta, wsum, lmv, lmi, flags, tid)) {
        for (int i = tid; i < 1 + 5 * A.L; i += kConsumers) A.counters[i] = 0;
        // every CTA has staged the LM head's input: the last down's sums start the next step clear
        for (int64_t e = tid; e < (int64_t)M * A.H; e += kConsumers) A.fx_d[e] = 0;
      }
    }
  }
  __syncthreads();
  if (tid == 0) ring_drain(R, flags[0], A.err);
}

struct StepPlan {
  int grid, nst, splits, kmax, smem, o_merge;
  int64_t chunk;
  int smax[K_KINDS];
  int64_t total[K_KINDS];
  int64_t off_counters, off_abort, off_tickets, off_lm_ticket, off_cta_val, off_cta_idx, off_partials, off_attn_acc,
      off_attn_ml, off_attn_tickets, off_xb, off_fx_o, off_fx_d, off_fx_q, bytes;
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
  const int fixed = step_layout((int)B, p->kmax, 0).total;
  int nst = (227 * 1024 - fixed) / (kBlockBytes + 16);
  const int cap_st = env_int("QD_STEP_STAGES", 16);  // tuning: upper bound on the ring depth
  if (nst > cap_st) nst = cap_st;
  if (nst > 16) nst = 16;
  if (nst < 2) return set_error(QD_ERR_UNSUPPORTED, "step: shared memory too small for batch %lld", (long long)B);
  p->nst = nst;
  p->smem = step_layout((int)B, p->kmax, nst).total;
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
  p->off_xb = take(B * H * 2);
  p->off_fx_o = take(B * H * 8);
  p->off_fx_d = take(B * H * 8);
  p->off_fx_q = take(B * n_rows[K_QKV] * 8);
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

template <int M>
static int launch_step(const StepArgs& a, int smem, cudaStream_t stream) {
  auto kern = step_kernel<M>;
  if (int rc = set_max_dynamic_smem((const void*)kern, smem)) return rc;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
  if (e != cudaSuccess || per_sm < 1)
    return set_error(QD_ERR_UNSUPPORTED, "step kernel does not fit on an SM (smem %d B)", smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(kThreads);
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
  a.xb = reinterpret_cast<__nv_bfloat16*>(sc + p.off_xb);
  a.fx_o = reinterpret_cast<int64_t*>(sc + p.off_fx_o);
  a.fx_d = reinterpret_cast<int64_t*>(sc + p.off_fx_d);
  a.fx_q = reinterpret_cast<int64_t*>(sc + p.off_fx_q);
  switch (d->batch) {
    case 1: return launch_step<1>(a, p.smem, stream);
    case 2: return launch_step<2>(a, p.smem, stream);
    case 3: return launch_step<3>(a, p.smem, stream);
    case 4: return launch_step<4>(a, p.smem, stream);
    case 5: return launch_step<5>(a, p.smem, stream);
    case 6: return launch_step<6>(a, p.smem, stream);
    case 7: return launch_step<7>(a, p.smem, stream);
    case 8: return launch_step<8>(a, p.smem, stream);
  }
  return set_error(QD_ERR_UNSUPPORTED, "batch %lld", (long long)d->batch);
}
