// Persistent tcgen05 decode step for batches of 4..64 sequences, sm_100a: one cooperative launch per
// step, one CTA per SM, the same arithmetic and the same work partitions as the tensor-core kernel
// chain (qd_pack_act, qd_tc_*, qd_attn_decode_tc), so the two give bit-identical tokens and logits.
//
// Roles inside a CTA of 10 warps:
//   warps 0-7  consumers: RMSNorm packing of whole activation rows, the GEMM epilogues (tensor-memory
//              readout + split-K flush + fused epilogue), and on warps 0-3 the attention softmax and
//              merge;
//   warp 8     producer: the weight blocks of every projection of the step, back to back, into a ring
//              of (weight block + activation tile) stages; the activation tiles of an op go out once
//              that op's input is complete; the attention K/V by TMA into a second ring;
//   warp 9     MMA issuer: tcgen05.mma for the projections (swap-AB, M = 128 weight rows, N = the
//              padded batch) and for attention (q.k and P.V per 128-key chunk).
// Ops wait on release/acquire completion counters (bounded waits, shared abort flag); the CTA that
// completes the LM head's argmax clears the counters for the next step.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "qd_attn_dev.cuh"
#include "qd_gemv_dev.cuh"
#include "qd_plan.h"
#include "qd_umma.cuh"

namespace qd {

constexpr int kPThreads = 320;
constexpr int kPSoftBar = 2;              // named barrier of warps 0-3 (1 = all 256 consumers)
constexpr int kAKeys = 128;               // attention chunk (q.k MMA M)
constexpr int kABox = kAKeys * 128;       // one [128 keys][64 dims] BF16 box
constexpr int kAStage = 4 * kABox;        // K lo, K hi, V lo, V hi
constexpr int kAStages = 2;
constexpr int kAN = 16;                   // attention MMA N (4 heads + 12 zero rows)
constexpr int kAStageMax = 160;           // attention merge staging: 3 x 4 x smax floats
constexpr int kTmemCols = 256;            // GEMM accumulators [0, 2N), attention S [128, 160), O [160, 192)
enum { P_QKV = 0, P_O = 1, P_GU = 2, P_DOWN = 3, P_LM = 4, P_KINDS = 5 };

// counters: [0] embedded rows; layer l at 1 + 7l: +0 rows packed (ln1), +1 QKV groups, +2 attention
// pairs, +3 O groups, +4 rows packed (ln2), +5 gate/up groups, +6 down groups; then final-norm rows
struct alignas(64) TcStepArgs {
  CUtensorMap tk, tv;  // 5-D over the caches [L][B][nkv][cap][128], box {64, 128, 1, 1, 1}
  const char* w[P_KINDS];
  int64_t wlb[P_KINDS];
  int64_t wn[P_KINDS], wk[P_KINDS], total[P_KINDS];
  int smax[P_KINDS];
  const __nv_bfloat16 *ln1, *ln2, *qn, *kn, *fnorm;
  int L, H, I, nq, nkv, m_act, grid, nst, asmax;
  int64_t vocab;
  float eps, scale;
  int64_t* tok;
  int64_t* pos;
  __nv_bfloat16 *x, *q, *kc, *vc;
  int64_t c_ls, cs_b, cs_h, cap;
  const __nv_bfloat16 *cos, *sin;
  __nv_bfloat16* logits;
  int64_t ld_logits;
  __nv_bfloat16 *xh, *xa, *xi;  // packed activation operands ([k/64][N][64])
  int* err;
  int* abort_flag;
  int* counters;
  float* partials;
  int* tickets;
  float* cta_val;
  int* cta_idx;
  int* lm_ticket;
  float *apart_acc, *apart_ml;
  int* atickets;
  // The O and down projections leave fixed-point group sums ([M][H] int64) and the packer of each row
  // applies the residual add (x row += sums) before normalising it - no last-arriving CTA's reduction
  // between the projection and the next op
  int64_t *fx_o, *fx_d;
  uint64_t* trace;
};

struct TcStepLayout {
  int stage, gring, areg, qb, pb, stg, wsum, lmv, lmi, flags, aux, ared, bars, misc, total;
};

__host__ __device__ inline int tsal(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline TcStepLayout tc_step_layout(int N, int nst) {
  TcStepLayout L;
  L.stage = kBlockBytes + N * 128;
  L.gring = 0;
  int off = nst * L.stage;
  L.areg = tsal(off, 1024);  // attention K/V ring; the GEMM epilogue's `red` aliases its start
  off = L.areg + kAStages * kAStage;
  L.qb = off;                // [2 dim halves][16 rows][128 B]
  off += 2 * kAN * 128;
  L.pb = off;                // [2 buffers][2 key halves][16 rows][128 B]
  off += 2 * 2 * kAN * 128;
  L.stg = off;
  off += 3 * kGroup * kAStageMax * 4;
  L.wsum = off;
  off += N * kConsumerWarps * 4 + 64;
  L.lmv = off;
  off += tsal(N * 4, 16);
  L.lmi = off;
  off += tsal(N * 4, 16);
  L.flags = off;
  off += 16;
  L.aux = off;
  off += 512 * 4;
  L.ared = off;
  off += 3 * 16 * 4;
  L.bars = tsal(off, 8);
  off = L.bars + (2 * nst + 4 + 2 * kAStages + 8 + 2) * 8;
  L.misc = off;
  off += 16;
  L.total = tsal(off, 1024);
  return L;
}

__device__ __forceinline__ int* pctr(const TcStepArgs& A, int l, int op) { return A.counters + 1 + 7 * l + op; }
__device__ __forceinline__ int* final_pack_ctr(const TcStepArgs& A) { return A.counters + 1 + 7 * A.L; }

__device__ __forceinline__ void tstamp(const TcStepArgs& A, int cta, int op, int what, int tid) {
  if (A.trace && tid == 0) A.trace[((int64_t)cta * (3 + 7 * A.L) + op) * 4 + what] = globaltimer();
}

// One thread waits (bounded) until *cnt >= target; on expiry it flags the error and the abort flag.
__device__ bool poll_ctr(const TcStepArgs& A, const int* cnt, int target) {
  return wait_count_ge(cnt, target, A.abort_flag, A.err, kErrDep);
}
// ... and the 256 consumers proceed together
__device__ void wait_consumers(const TcStepArgs& A, const int* cnt, int target, int tid) {
  if (tid == 0) poll_ctr(A, cnt, target);
  named_bar(kBarConsumers, kConsumers);
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w, int v,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint32_t sw128(int row, int col) {
  return (uint32_t)(row * 128 + ((((col >> 3) ^ (row & 7)) & 7) << 4) + ((col & 7) << 1));
}

template <int N>
__device__ GemvArgs pop(const TcStepArgs& A, int kind, int l) {
  GemvArgs a = {};
  a.w = A.w[kind] + (int64_t)l * A.wlb[kind];
  a.n = A.wn[kind];
  a.n_valid = A.wn[kind];
  a.k = A.wk[kind];
  a.kblocks = (int)(A.wk[kind] / kBlockCols);
  a.total = A.total[kind];
  a.grid = A.grid;
  a.nst = A.nst;
  a.m_act = A.m_act;
  a.partials = A.partials;
  a.tickets = A.tickets;
  a.smax = A.smax[kind];
  a.err = A.err;
  a.eps = A.eps;
  if (kind == P_QKV) {
    a.x_packed = reinterpret_cast<const char*>(A.xh);
    a.q_norm = A.qn + (int64_t)l * 128;
    a.k_norm = A.kn + (int64_t)l * 128;
    a.cos = A.cos;
    a.sin = A.sin;
    a.pos = A.pos;
    a.cap = A.cap;
    a.nq = A.nq;
    a.nkv = A.nkv;
    a.q_out = A.q;
    a.k_cache = A.kc + (int64_t)l * A.c_ls;
    a.v_cache = A.vc + (int64_t)l * A.c_ls;
    a.cs_b = A.cs_b;
    a.cs_h = A.cs_h;
    a.done = pctr(A, l, 1);
  } else if (kind == P_O || kind == P_DOWN) {
    a.x_packed = reinterpret_cast<const char*>(kind == P_O ? A.xa : A.xi);
    a.out = A.x;
    a.ldo = A.H;
    a.res = A.x;
    a.ldr = A.H;
    a.fx = kind == P_O ? A.fx_o : A.fx_d;
    a.fx_ctr = pctr(A, l, kind == P_O ? 3 : 6);
  } else if (kind == P_GU) {
    a.x_packed = reinterpret_cast<const char*>(A.xh);
    a.out = A.xi;
    a.out_npad = N;
    a.done = pctr(A, l, 5);
  } else {
    a.x_packed = reinterpret_cast<const char*>(A.xh);
    a.n_valid = A.vocab;
    a.tok = A.tok;
    a.pos_inc = A.pos;
    a.inc_pos = 1;
    a.logits = A.logits;
    a.ld_logits = A.ld_logits;
    a.cta_val = A.cta_val;
    a.cta_idx = A.cta_idx;
    a.lm_ticket = A.lm_ticket;
  }
  return a;
}

// ------------------------------------------------------------------ roles
struct ProdState {
  int slot, round, issued;     // GEMM ring
  int aslot, around, aissued;  // attention ring
};
struct MmaState {
  int slot, fph, buf, uses0, uses1;  // GEMM ring / accumulators
  int agi, qph;                      // attention chunks issued so far, q-ready phases waited
};

// Producer lane: this CTA's blocks of one projection. Weight copies are gated only by free slots; the
// activation tiles wait (bounded) for the op's input counter, deferred for at most a ring's worth.
template <int N>
__device__ bool produce_gemm(const TcStepArgs& A, const GemvArgs& op, const int* in_ctr, int in_target, int cta,
                             char* smem, const TcStepLayout& Ly, uint32_t bars, ProdState& st, uint64_t pol) {
  const int nst = A.nst;
  const int64_t xt = (int64_t)N * 128;
  const int64_t b0 = part_begin(op.total, op.grid, cta), b1 = part_begin(op.total, op.grid, cta + 1);
  const int nblk = (int)(b1 - b0);
  const char* wsrc = op.w + b0 * (int64_t)kBlockBytes;
  int kb = (int)(b0 % op.kblocks);
  bool ready = false;
  int pslot[16], pkb[16], np = 0;
  for (int i = 0; i < nblk; ++i) {
    const uint32_t full = bars + 8u * st.slot, empty = bars + 8u * (nst + st.slot);
    if (st.round > 0 && !mbar_wait_abort(empty, (st.round - 1) & 1, A.err, kErrWaitEmpty, A.abort_flag)) return false;
    char* stage = smem + Ly.gring + st.slot * Ly.stage;
    mbar_arrive_expect_tx(full, (uint32_t)(kBlockBytes + xt));
    bulk_g2s(smem_u32(stage), wsrc + (int64_t)i * kBlockBytes, kBlockBytes, full, pol);
    if (ready) {
      bulk_g2s(smem_u32(stage + kBlockBytes), op.x_packed + kb * xt, (uint32_t)xt, full, pol);
    } else {
      pslot[np] = st.slot;
      pkb[np++] = kb;
      if (np == nst || i == nblk - 1) {
        if (!poll_ctr(A, in_ctr, in_target)) return false;
        fence_proxy_async_global();  // the operand was written with ordinary stores by other CTAs
        ready = true;
        for (int j = 0; j < np; ++j)
          bulk_g2s(smem_u32(smem + Ly.gring + pslot[j] * Ly.stage + kBlockBytes), op.x_packed + pkb[j] * xt,
                   (uint32_t)xt, bars + 8u * pslot[j], pol);
        np = 0;
      }
    }
    ++st.issued;
    if (++kb == op.kblocks) kb = 0;
    if (++st.slot == nst) {
      st.slot = 0;
      ++st.round;
    }
  }
  return true;
}

template <int N>
__device__ void mma_gemm(const TcStepArgs& A, const GemvArgs& op, int cta, char* smem, const TcStepLayout& Ly,
                         uint32_t bars, uint32_t tmem, MmaState& ms, bool& ok) {
  const int nst = A.nst;
  const uint32_t idesc = umma_idesc_bf16(N);
  const uint32_t accf0 = bars + 8u * (2 * nst), acce0 = bars + 8u * (2 * nst + 2);
  const int64_t b0 = part_begin(op.total, op.grid, cta), b1 = part_begin(op.total, op.grid, cta + 1);
  const int nblk = (int)(b1 - b0);
  int kb = (int)(b0 % op.kblocks);
  for (int i = 0; i < nblk; ++i) {
    const bool seg_start = (i == 0) || (kb == 0);
    const bool seg_end = (kb == op.kblocks - 1) || (i == nblk - 1);
    const int uses = ms.buf ? ms.uses1 : ms.uses0;
    if (seg_start && uses > 0 && ok) ok = mbar_wait_abort(acce0 + 8u * ms.buf, (uses - 1) & 1, A.err, kErrWaitFull, A.abort_flag);
    if (ok) ok = mbar_wait_abort(bars + 8u * ms.slot, ms.fph, A.err, kErrWaitFull, A.abort_flag);
    tc_fence_after();
    if (ok) {
      const uint32_t sa = smem_u32(smem + Ly.gring + ms.slot * Ly.stage), sb = sa + kBlockBytes;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        umma_bf16(tmem + ms.buf * N, umma_desc_sw128(sa + 32 * j), umma_desc_sw128(sb + 32 * j), idesc,
                  (seg_start && j == 0) ? 0u : 1u);
    }
    umma_commit(bars + 8u * (nst + ms.slot));
    if (seg_end) {
      umma_commit(accf0 + 8u * ms.buf);
      if (ms.buf) ++ms.uses1; else ++ms.uses0;
      ms.buf ^= 1;
    }
    if (++ms.slot == nst) {
      ms.slot = 0;
      ms.fph ^= 1;
    }
    if (++kb == op.kblocks) kb = 0;
  }
}

template <int N, int MODE, bool DEFER = false>
__device__ void epilogue_gemm(const TcStepArgs& A, const GemvArgs& op, int cta, char* smem, const TcStepLayout& Ly,
                              uint32_t bars, uint32_t tmem, int& buf, int (&fph)[2], int tid) {
  const int nst = A.nst, warp = tid >> 5, lane = tid & 31;
  const uint32_t accf0 = bars + 8u * (2 * nst), acce0 = bars + 8u * (2 * nst + 2);
  float* red = reinterpret_cast<float*>(smem + Ly.areg);
  float* wsum = reinterpret_cast<float*>(smem + Ly.wsum);
  float* lmv = reinterpret_cast<float*>(smem + Ly.lmv);
  int* lmi = reinterpret_cast<int*>(smem + Ly.lmi);
  int* flags = reinterpret_cast<int*>(smem + Ly.flags);
  float* aux = reinterpret_cast<float*>(smem + Ly.aux);
  if constexpr (MODE == MODE_QKV) qkv_prologue(op, aux, flags, tid);
  if constexpr (MODE == MODE_LM) {
    if (tid < N) {
      lmv[tid] = -INFINITY;
      lmi[tid] = 0x7fffffff;
    }
    named_bar(kBarConsumers, kConsumers);
  }
  bool ok = true;
  const int q = warp & 3, half = warp >> 2;
  const int64_t b0 = part_begin(op.total, op.grid, cta), b1 = part_begin(op.total, op.grid, cta + 1);
  int64_t seg_first = b0;
  int g = (int)(b0 / op.kblocks);
  int kb = (int)(b0 % op.kblocks) - 1;
  for (int64_t b = b0; b < b1; ++b) {
    if (++kb == op.kblocks) {
      kb = 0;
      ++g;
    }
    const bool seg_end = (kb == op.kblocks - 1) || (b == b1 - 1);
    if (!seg_end) continue;
    if (ok) ok = mbar_wait_abort(accf0 + 8u * buf, fph[buf], A.err, kErrWaitFull, A.abort_flag);
    fph[buf] ^= 1;
    tc_fence_after();
#pragma unroll
    for (int c8 = 0; c8 < N / 16; ++c8) {
      float v[8];
      const int col = half * (N / 2) + 8 * c8;
      tmem_ld8(tmem + ((uint32_t)(32 * q) << 16) + buf * N + col, v);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 8; ++e) red[(col + e) * kBlockRows + 32 * q + lane] = v[e];
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(acce0 + 8u * buf);
    buf ^= 1;
    named_bar(kBarConsumers, kConsumers);
    flush_segment<N, MODE, DEFER>(op, g, seg_first, b, cta, red, wsum, lmv, lmi, aux, flags, tid);
    seg_first = b + 1;
  }
  if constexpr (MODE == MODE_LM) {
    if (lm_global_argmax<N>(op, cta, wsum, lmv, lmi, flags, tid)) {
      for (int i = tid; i < 2 + 7 * A.L; i += kConsumers) A.counters[i] = 0;  // the next step starts clean
    }
  }
}

// RMSNorm of whole activation rows (this CTA's rows cta, cta + G, ...) into the packed operand,
// qd_pack_act's arithmetic (256 threads). Signals one count per row. With fxs (a residual projection's
// fixed-point sums), each row first gets the projection's RES epilogue, x = bf16(x + bf16(sum)), written
// back to x in place (this CTA is the row's only reader), and its sums are cleared for the next use.
__device__ void pack_rows_norm(const TcStepArgs& A, const __nv_bfloat16* norm_w, int* ctr, int npad, int cta,
                               float* wsum, int tid, int64_t* fxs = nullptr) {
  const int warp = tid >> 5, lane = tid & 31;
  const int k8 = A.H >> 3;
  for (int m = cta; m < A.m_act; m += A.grid) {
    float sq = 0.f;
    for (int qq = tid; qq < k8; qq += kConsumers) {
      uint4 v = ld_cg_v4(A.x + (int64_t)m * A.H + qq * 8);
      if (fxs) {
        longlong2* sp = reinterpret_cast<longlong2*>(fxs + (int64_t)m * A.H + qq * 8);
        const longlong2 sv[4] = {__ldcg(sp), __ldcg(sp + 1), __ldcg(sp + 2), __ldcg(sp + 3)};
        const uint32_t ru[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float lo = bf16r(bf_lo(ru[e]) + bf16r(fx_to_float(sv[e].x)));
          const float hi = bf16r(bf_hi(ru[e]) + bf16r(fx_to_float(sv[e].y)));
          o[e] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
        }
        v = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(A.x + (int64_t)m * A.H + qq * 8) = v;  // re-read below by this thread
#pragma unroll
        for (int e = 0; e < 4; ++e) sp[e] = make_longlong2(0, 0);
      }
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = bf_lo(u[e]), hi = bf_hi(u[e]);
        sq = fmaf(lo, lo, sq);
        sq = fmaf(hi, hi, sq);
      }
    }
    sq = warp_sum(sq);
    if (lane == 0) wsum[warp] = sq;
    named_bar(kBarConsumers, kConsumers);
    float ss = 0.f;
#pragma unroll
    for (int w8 = 0; w8 < 8; ++w8) ss += wsum[w8];
    const float rstd = 1.0f / sqrtf(ss / (float)A.H + A.eps);
    for (int qq = tid; qq < k8; qq += kConsumers) {
      const uint4 v = ld_cg_v4(A.x + (int64_t)m * A.H + qq * 8);
      const uint4 wv = *reinterpret_cast<const uint4*>(norm_w + qq * 8);
      const uint32_t xu[4] = {v.x, v.y, v.z, v.w};
      const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = bf16r(bf_lo(wu[e]) * bf16r(bf_lo(xu[e]) * rstd));
        const float hi = bf16r(bf_hi(wu[e]) * bf16r(bf_hi(xu[e]) * rstd));
        o[e] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
      }
      const int kb = qq >> 3, c = qq & 7;
      *reinterpret_cast<uint4*>(A.xh + ((int64_t)kb * npad + m) * 64 + ((c ^ (m & 7)) << 3)) =
          make_uint4(o[0], o[1], o[2], o[3]);
    }
    signal_done(ctr, tid);  // barrier, then one release increment
  }
}

// ------------------------------------------------------------------ attention roles (one layer)
struct AttnWork {
  int64_t len, T;
  int nch, G, n, pair0, ci0;
};

__device__ __forceinline__ AttnWork attn_work(const TcStepArgs& A, int64_t len, int cta) {
  AttnWork w;
  w.len = len;
  w.nch = (int)((len + kAKeys - 1) / kAKeys);
  w.T = (int64_t)A.m_act * A.nkv * w.nch;
  w.G = (int)(w.T < A.grid ? w.T : A.grid);
  w.n = 0;
  w.pair0 = 0;
  w.ci0 = 0;
  if (cta < w.G) {
    const int64_t c0 = part_begin(w.T, w.G, cta), c1 = part_begin(w.T, w.G, cta + 1);
    w.n = (int)(c1 - c0);
    w.pair0 = (int)(c0 / w.nch);
    w.ci0 = (int)(c0 - (int64_t)w.pair0 * w.nch);
  }
  return w;
}

__device__ bool produce_attn(const TcStepArgs& A, const AttnWork& w, int l, const TcStepLayout& Ly, uint32_t sbase,
                             uint32_t abars, ProdState& st, uint64_t pol) {
  int pair = w.pair0, ci = w.ci0;
  for (int i = 0; i < w.n; ++i) {
    const uint32_t full = abars + 8u * st.aslot, empty = abars + 8u * (kAStages + st.aslot);
    if (st.around > 0 && !mbar_wait_abort(empty, (st.around - 1) & 1, A.err, kErrWaitEmpty, A.abort_flag)) return false;
    if (ci == w.nch - 1) {  // this chunk holds the new key, appended by the QKV epilogue
      if (!poll_ctr(A, pctr(A, l, 1), A.nq + 2 * A.nkv)) return false;
      fence_proxy_async_global();
    }
    const int b = pair / A.nkv, kvh = pair - b * A.nkv, k0 = ci * kAKeys;
    const uint32_t st_addr = sbase + Ly.areg + st.aslot * kAStage;
    mbar_arrive_expect_tx(full, kAStage);
    tma_load_5d(st_addr, &A.tk, 0, k0, kvh, b, l, full, pol);
    tma_load_5d(st_addr + kABox, &A.tk, 64, k0, kvh, b, l, full, pol);
    tma_load_5d(st_addr + 2 * kABox, &A.tv, 0, k0, kvh, b, l, full, pol);
    tma_load_5d(st_addr + 3 * kABox, &A.tv, 64, k0, kvh, b, l, full, pol);
    ++st.aissued;
    if (++ci == w.nch) {
      ci = 0;
      ++pair;
    }
    if (++st.aslot == kAStages) {
      st.aslot = 0;
      ++st.around;
    }
  }
  return true;
}

__device__ void mma_attn(const TcStepArgs& A, const AttnWork& w, const TcStepLayout& Ly, uint32_t sbase,
                         uint32_t abars, uint32_t tS0, uint32_t tO0, MmaState& ms, bool& ok) {
  const uint32_t id_qk = umma_idesc_bf16(kAN, false), id_pv = umma_idesc_bf16(kAN, true);
  auto afull = [&](int s) { return abars + 8u * s; };
  auto aempty = [&](int s) { return abars + 8u * (kAStages + s); };
  auto sfull = [&](int b) { return abars + 8u * (2 * kAStages + b); };
  auto pfull = [&](int b) { return abars + 8u * (2 * kAStages + 2 + b); };
  auto ofull = [&](int b) { return abars + 8u * (2 * kAStages + 4 + b); };
  auto dfree = [&](int b) { return abars + 8u * (2 * kAStages + 6 + b); };
  const uint32_t qready = abars + 8u * (2 * kAStages + 8);
  int ci_next = w.ci0;
  auto issue_qk = [&](int i) {
    const int gi = ms.agi + i, slot = gi % kAStages, b = gi & 1;
    if (ok) ok = mbar_wait_abort(afull(slot), (gi / kAStages) & 1, A.err, kErrWaitFull, A.abort_flag);
    if (ok && gi >= 2) ok = mbar_wait_abort(dfree(b), ((gi >> 1) - 1) & 1, A.err, kErrWaitFull, A.abort_flag);
    if (ok && (i == 0 || ci_next == 0)) {  // a pair segment starts: its q must be in place
      ok = mbar_wait_abort(qready, ms.qph & 1, A.err, kErrWaitFull, A.abort_flag);
      ++ms.qph;
    }
    tc_fence_after();
    if (ok) {
      const uint32_t stg = sbase + Ly.areg + slot * kAStage;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        umma_bf16(tS0 + b * kAN, umma_desc_sw128(stg + (j >> 2) * kABox + (j & 3) * 32),
                  umma_desc_sw128(sbase + Ly.qb + (j >> 2) * (kAN * 128) + (j & 3) * 32), id_qk, j > 0 ? 1u : 0u);
    }
    umma_commit(sfull(b));
    if (++ci_next == w.nch) ci_next = 0;
  };
  if (w.n > 0) issue_qk(0);
  for (int i = 0; i < w.n; ++i) {
    const bool next_new_pair = (i + 1 < w.n) && ci_next == 0;  // its q.k waits for the pair's q: after P.V
    if (i + 1 < w.n && !next_new_pair) issue_qk(i + 1);
    const int gi = ms.agi + i, slot = gi % kAStages, b = gi & 1;
    if (ok) ok = mbar_wait_abort(pfull(b), (gi >> 1) & 1, A.err, kErrWaitFull, A.abort_flag);
    tc_fence_after();
    if (ok) {
      const uint32_t vst = sbase + Ly.areg + slot * kAStage + 2 * kABox;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        umma_bf16(tO0 + b * kAN, umma_desc_sw128(vst + j * 2048, kABox, 1024),
                  umma_desc_sw128(sbase + Ly.pb + b * (2 * kAN * 128) + (j >> 2) * (kAN * 128) + (j & 3) * 32), id_pv,
                  j > 0 ? 1u : 0u);
    }
    umma_commit(ofull(b));
    umma_commit(aempty(slot));
    if (next_new_pair) issue_qk(i + 1);
  }
  ms.agi += w.n;
}

// Softmax + epilogue on warps 0-3 (tid 0..127): the attention output of each pair goes straight into
// the O projection's packed operand; one count per finished pair.
__device__ void softmax_attn(const TcStepArgs& A, const AttnWork& w, int l, int cta, char* smem,
                             const TcStepLayout& Ly, uint32_t abars, uint32_t tS0, uint32_t tO0, int& agi, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  auto sfull = [&](int b) { return abars + 8u * (2 * kAStages + b); };
  auto pfull = [&](int b) { return abars + 8u * (2 * kAStages + 2 + b); };
  auto ofull = [&](int b) { return abars + 8u * (2 * kAStages + 4 + b); };
  auto dfree = [&](int b) { return abars + 8u * (2 * kAStages + 6 + b); };
  const uint32_t qready = abars + 8u * (2 * kAStages + 8);
  float* red = reinterpret_cast<float*>(smem + Ly.ared);
  const int N = (A.m_act + 15) / 16 * 16;
  int pair = w.pair0, ci = w.ci0, seg_first = ci;
  float m_run[kGroup], l_thr[kGroup], acc[kGroup];
  // q of a pair (written every layer by other CTAs: read through L2) is loaded one pair ahead
  const int pair_last = w.n > 0 ? w.pair0 + (w.ci0 + w.n - 1) / w.nch : 0;
  unsigned short qn[kGroup];
  auto load_q = [&](int pr) {
    const int b = pr / A.nkv, kvh = pr - b * A.nkv;
#pragma unroll
    for (int h = 0; h < kGroup; ++h)
      qn[h] = __ldcg(reinterpret_cast<const unsigned short*>(A.q) + ((int64_t)b * A.nq + kvh * kGroup + h) * kHeadDim +
                     tid);
  };
  auto put_q = [&](int pr) {
#pragma unroll
    for (int h = 0; h < kGroup; ++h)
      *reinterpret_cast<unsigned short*>(smem + Ly.qb + (tid >> 6) * (kAN * 128) + sw128(h, tid & 63)) = qn[h];
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(qready);
    if (pr + 1 <= pair_last) load_q(pr + 1);
  };
  auto reset = [&]() {
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      m_run[h] = -INFINITY;
      l_thr[h] = 0.f;
      acc[h] = 0.f;
    }
  };
  auto out_index = [&](int b, int hq, int d) {
    const int k = hq * kHeadDim + d, kb = k >> 6, c = k & 63;
    return ((int64_t)kb * N + b) * 64 + (((c >> 3) ^ (b & 7)) << 3) + (c & 7);
  };
  if (w.n > 0) {
    load_q(pair);
    put_q(pair);
  }
  reset();
  bool ok = true;
  for (int i = 0; i < w.n; ++i) {
    const int gi = agi + i, slot = gi % kAStages, b = gi & 1;
    const int k0 = ci * kAKeys;
    const int nk = (int)((w.len - k0) < kAKeys ? (w.len - k0) : kAKeys);
    if (ok) ok = mbar_wait_abort(sfull(b), (gi >> 1) & 1, A.err, kErrWaitFull, A.abort_flag);
    tc_fence_after();
    float s[4];
    tmem_ld4(tS0 + b * kAN + ((uint32_t)(32 * warp) << 16), s);
    tmem_wait_ld();
    const bool valid = tid < nk;
    float mx[kGroup];
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      s[h] = valid ? s[h] * A.scale : -INFINITY;
      mx[h] = warp_max(s[h]);
    }
    float* rb = red + (gi & 1) * 16;
    if (lane == 0) {
#pragma unroll
      for (int h = 0; h < kGroup; ++h) rb[warp * 4 + h] = mx[h];
    }
    named_bar(kPSoftBar, 128);
    float alpha[kGroup];
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      const float mc = fmaxf(fmaxf(rb[h], rb[4 + h]), fmaxf(rb[8 + h], rb[12 + h]));
      const float m_new = fmaxf(m_run[h], mc);
      alpha[h] = expf(m_run[h] - m_new);
      const float p = valid ? expf(s[h] - m_new) : 0.f;
      l_thr[h] = l_thr[h] * alpha[h] + p;
      m_run[h] = m_new;
      *reinterpret_cast<__nv_bfloat16*>(smem + Ly.pb + b * (2 * kAN * 128) + (tid >> 6) * (kAN * 128) +
                                        sw128(h, tid & 63)) = __float2bfloat16_rn(p);
    }
    if (nk < kAKeys) {  // V rows past the valid length: zero for P.V
      char* vst = smem + Ly.areg + slot * kAStage + 2 * kABox;
      for (int r = nk + tid; r < kAKeys; r += 128)
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          *reinterpret_cast<uint4*>(vst + r * 128 + 16 * c) = make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(vst + kABox + r * 128 + 16 * c) = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(pfull(b));
    const bool pair_end = (ci == w.nch - 1) || (i == w.n - 1);
    if (pair_end && i + 1 < w.n) put_q(pair + 1);
    if (ok) ok = mbar_wait_abort(ofull(b), (gi >> 1) & 1, A.err, kErrWaitFull, A.abort_flag);
    tc_fence_after();
    float o[4];
    tmem_ld4(tO0 + b * kAN + ((uint32_t)(32 * warp) << 16), o);
    tmem_wait_ld();
#pragma unroll
    for (int h = 0; h < kGroup; ++h) acc[h] = fmaf(acc[h], alpha[h], o[h]);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(dfree(b));
    if (pair_end) {
      float lsum[kGroup];
#pragma unroll
      for (int h = 0; h < kGroup; ++h) lsum[h] = warp_sum(l_thr[h]);
      float* lb = red + 32;
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < kGroup; ++h) lb[warp * 4 + h] = lsum[h];
      }
      named_bar(kPSoftBar, 128);
#pragma unroll
      for (int h = 0; h < kGroup; ++h) lsum[h] = ((lb[h] + lb[4 + h]) + lb[8 + h]) + lb[12 + h];
      const int bb = pair / A.nkv, kvh = pair - bb * A.nkv;
      bool wrote = false;
      if (seg_first == 0 && ci == w.nch - 1) {
#pragma unroll
        for (int h = 0; h < kGroup; ++h)
          A.xa[out_index(bb, kvh * kGroup + h, tid)] = __float2bfloat16_rn(acc[h] / lsum[h]);
        wrote = true;
      } else {
        const int64_t gc0 = (int64_t)pair * w.nch;
        const int c_lo = part_owner(w.T, w.G, gc0);
        const int pslot = cta - c_lo;
        const int nseg = part_owner(w.T, w.G, gc0 + w.nch - 1) - c_lo + 1;
        if (pslot < 0 || pslot >= A.asmax || nseg > A.asmax) {
          if (tid == 0) atomicOr(A.err, kErrDep);
        } else {
          const int64_t prow = ((int64_t)pair * A.asmax + pslot) * kGroup;
#pragma unroll
          for (int h = 0; h < kGroup; ++h) __stcg(A.apart_acc + (prow + h) * kHeadDim + tid, acc[h]);
          if (tid < 2 * kGroup) __stcg(A.apart_ml + prow * 2 + tid, (tid & 1) ? lsum[tid >> 1] : m_run[tid >> 1]);
          named_bar(kPSoftBar, 128);
          int* flag = reinterpret_cast<int*>(smem + Ly.misc + 4);
          if (tid == 0) {
            const int cnt = ci - seg_first + 1;
            *flag = (atom_add_acq_rel(A.atickets + pair, cnt) + cnt == w.nch) ? 1 : 0;
          }
          named_bar(kPSoftBar, 128);
          if (*flag) {
            float* mm = reinterpret_cast<float*>(smem + Ly.stg);
            float* ll = mm + kGroup * nseg;
            float* ww = ll + kGroup * nseg;
            const int64_t prow0 = (int64_t)pair * A.asmax * kGroup;
            for (int t = tid; t < kGroup * nseg; t += 128) {
              const int h = t / nseg, sg = t - h * nseg;
              mm[t] = ld_cg_f32(A.apart_ml + (prow0 + (int64_t)sg * kGroup + h) * 2);
              ll[t] = ld_cg_f32(A.apart_ml + (prow0 + (int64_t)sg * kGroup + h) * 2 + 1);
            }
            named_bar(kPSoftBar, 128);
            for (int t = tid; t < kGroup * nseg; t += 128) {
              const int h = t / nseg;
              float m2 = -INFINITY;
              for (int sg = 0; sg < nseg; ++sg) m2 = fmaxf(m2, mm[h * nseg + sg]);
              ww[t] = (mm[t] == -INFINITY) ? 0.f : expf(mm[t] - m2);
            }
            named_bar(kPSoftBar, 128);
#pragma unroll
            for (int h = 0; h < kGroup; ++h) {
              float nm = 0.f;
              for (int s0 = 0; s0 < nseg; s0 += 8) {
                float av[8];
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  av[j] = (s0 + j < nseg)
                              ? ld_cg_f32(A.apart_acc + (prow0 + (int64_t)(s0 + j) * kGroup + h) * kHeadDim + tid)
                              : 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  if (s0 + j < nseg) nm = fmaf(av[j], ww[h * nseg + s0 + j], nm);
              }
              float den = 0.f;
              for (int sg = 0; sg < nseg; ++sg) den = fmaf(ll[h * nseg + sg], ww[h * nseg + sg], den);
              A.xa[out_index(bb, kvh * kGroup + h, tid)] = __float2bfloat16_rn(nm / den);
            }
            if (tid == 0) atomicExch(A.atickets + pair, 0);
            wrote = true;
          }
        }
      }
      fence_proxy_async_global();  // the O projection's bulk copies read these outputs
      named_bar(kPSoftBar, 128);   // outputs stored (and staging / sums free) before the release
      if (wrote && tid == 0) red_release_add(pctr(A, l, 2), 1);
      if (++ci == w.nch) {
        ci = 0;
        ++pair;
      }
      seg_first = ci;
      reset();
    } else {
      ++ci;
    }
  }
  agi += w.n;
}

// ------------------------------------------------------------------ the step kernel
template <int N>
__global__ void __launch_bounds__(kPThreads, 1) tc_step_kernel(const __grid_constant__ TcStepArgs A) {
  extern __shared__ __align__(1024) char smem_raw[];
  char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const TcStepLayout Ly = tc_step_layout(N, A.nst);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  const int nst = A.nst;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + Ly.bars;                 // gfull[nst], gempty[nst], accf[2], acce[2]
  const uint32_t abars = bars + 8u * (2 * nst + 4);      // afull[2], aempty[2], sfull, pfull, ofull, dfree, qready
  const uint32_t aregfree = abars + 8u * (2 * kAStages + 9);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + Ly.misc);
  int* issued_s = reinterpret_cast<int*>(smem + Ly.misc + 8);

  if (tid == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(bars + 8u * s, 1);
      mbar_init(bars + 8u * (nst + s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bars + 8u * (2 * nst + i), 1);
      mbar_init(bars + 8u * (2 * nst + 2 + i), kConsumerWarps);
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(abars + 8u * s, 1);
      mbar_init(abars + 8u * (kAStages + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(abars + 8u * (2 * kAStages + b), 1);      // sfull
      mbar_init(abars + 8u * (2 * kAStages + 2 + b), 4);  // pfull
      mbar_init(abars + 8u * (2 * kAStages + 4 + b), 1);  // ofull
      mbar_init(abars + 8u * (2 * kAStages + 6 + b), 4);  // dfree
    }
    mbar_init(abars + 8u * (2 * kAStages + 8), 4);  // qready
    mbar_init(aregfree, 1);
    fence_mbar_init();
    issued_s[0] = 0;
    issued_s[1] = 0;
  }
  if (warp == 9) tmem_alloc(smem_u32(tslot), kTmemCols);
  if (warp < 4) {  // q and P operand tiles start zero (rows 4..15 are the padded heads)
    for (int i = tid; i < (Ly.stg - Ly.qb) / 16; i += 128)
      *reinterpret_cast<uint4*>(smem + Ly.qb + 16 * i) = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tS0 = tmem + 128, tO0 = tmem + 128 + 2 * kAN;
  const int64_t pos = ld_cg_s64(A.pos);
  const int64_t len = attn_len_at(pos, A.cap, A.err, tid == 0 && cta == 0);
  const AttnWork aw = attn_work(A, len, cta);
  const int M = A.m_act;

  if (warp == 8) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      ProdState st = {0, 0, 0, 0, 0, 0};
      bool ok = true;
      for (int l = 0; l < A.L && ok; ++l) {
        ok = produce_gemm<N>(A, pop<N>(A, P_QKV, l), pctr(A, l, 0), M, cta, smem, Ly, bars, st, pol);
        if (ok && aw.n > 0) ok = mbar_wait_abort(aregfree, l & 1, A.err, kErrWaitEmpty, A.abort_flag) &&
                                 produce_attn(A, aw, l, Ly, sbase, abars, st, pol);
        if (ok) ok = produce_gemm<N>(A, pop<N>(A, P_O, l), pctr(A, l, 2), M * A.nkv, cta, smem, Ly, bars, st, pol);
        if (ok) ok = produce_gemm<N>(A, pop<N>(A, P_GU, l), pctr(A, l, 4), M, cta, smem, Ly, bars, st, pol);
        if (ok)
          ok = produce_gemm<N>(A, pop<N>(A, P_DOWN, l), pctr(A, l, 5), (int)(A.wn[P_GU] / kBlockRows), cta, smem, Ly,
                               bars, st, pol);
      }
      if (ok) produce_gemm<N>(A, pop<N>(A, P_LM, 0), final_pack_ctr(A), M, cta, smem, Ly, bars, st, pol);
      issued_s[0] = st.issued;
      issued_s[1] = st.aissued;
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      MmaState ms = {0, 0, 0, 0, 0, 0, 0};
      bool ok = true;
      for (int l = 0; l < A.L; ++l) {
        mma_gemm<N>(A, pop<N>(A, P_QKV, l), cta, smem, Ly, bars, tmem, ms, ok);
        mma_attn(A, aw, Ly, sbase, abars, tS0, tO0, ms, ok);
        mma_gemm<N>(A, pop<N>(A, P_O, l), cta, smem, Ly, bars, tmem, ms, ok);
        mma_gemm<N>(A, pop<N>(A, P_GU, l), cta, smem, Ly, bars, tmem, ms, ok);
        mma_gemm<N>(A, pop<N>(A, P_DOWN, l), cta, smem, Ly, bars, tmem, ms, ok);
      }
      mma_gemm<N>(A, pop<N>(A, P_LM, 0), cta, smem, Ly, bars, tmem, ms, ok);
    }
  } else {
    // ---------------------------------------------------------------- consumers (256 threads)
    float* wsum = reinterpret_cast<float*>(smem + Ly.wsum);
    int buf = 0, fph[2] = {0, 0}, agi = 0;
    // embedding: CTA i < M gathers row i of the tied, packed embedding
    if (cta < M) {
      int64_t t = ld_cg_s64(A.tok + cta);
      if (t < 0 || t >= A.vocab) {
        if (tid == 0) atomicOr(A.err, QD_DEVERR_TOKEN);
        t = t < 0 ? 0 : A.vocab - 1;
      }
      const int kb = A.H / kBlockCols;
      for (int q8 = tid; q8 < A.H / 8; q8 += kConsumers) {
        const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(A.w[P_LM]) +
                                                        packed_offset_elems(t, (int64_t)q8 * 8, kb));
        *reinterpret_cast<uint4*>(A.x + (int64_t)cta * A.H + q8 * 8) = v;
      }
      signal_done(A.counters, tid);
    }
    for (int l = 0; l < A.L; ++l) {
      wait_consumers(A, l == 0 ? A.counters : pctr(A, l - 1, 6), l == 0 ? M : (int)A.total[P_DOWN], tid);
      tstamp(A, cta, 1 + 7 * l, 0, tid);
      pack_rows_norm(A, A.ln1 + (int64_t)l * A.H, pctr(A, l, 0), N, cta, wsum, tid, l == 0 ? nullptr : A.fx_d);
      epilogue_gemm<N, MODE_QKV>(A, pop<N>(A, P_QKV, l), cta, smem, Ly, bars, tmem, buf, fph, tid);
      tstamp(A, cta, 2 + 7 * l, 0, tid);
      if (tid == 0) mbar_arrive(aregfree);  // `red` is free: the attention ring may fill
      wait_consumers(A, pctr(A, l, 1), A.nq + 2 * A.nkv, tid);
      if (warp < 4) softmax_attn(A, aw, l, cta, smem, Ly, abars, tS0, tO0, agi, tid);
      tstamp(A, cta, 3 + 7 * l, 0, tid);
      named_bar(kBarConsumers, kConsumers);  // the attention ring is drained before `red` is reused
      epilogue_gemm<N, MODE_RES, true>(A, pop<N>(A, P_O, l), cta, smem, Ly, bars, tmem, buf, fph, tid);
      tstamp(A, cta, 4 + 7 * l, 0, tid);
      wait_consumers(A, pctr(A, l, 3), (int)A.total[P_O], tid);
      pack_rows_norm(A, A.ln2 + (int64_t)l * A.H, pctr(A, l, 4), N, cta, wsum, tid, A.fx_o);
      epilogue_gemm<N, MODE_SWIGLU>(A, pop<N>(A, P_GU, l), cta, smem, Ly, bars, tmem, buf, fph, tid);
      tstamp(A, cta, 5 + 7 * l, 0, tid);
      epilogue_gemm<N, MODE_RES, true>(A, pop<N>(A, P_DOWN, l), cta, smem, Ly, bars, tmem, buf, fph, tid);
      tstamp(A, cta, 6 + 7 * l, 0, tid);
    }
    wait_consumers(A, pctr(A, A.L - 1, 6), (int)A.total[P_DOWN], tid);
    pack_rows_norm(A, A.fnorm, final_pack_ctr(A), N, cta, wsum, tid, A.fx_d);
    epilogue_gemm<N, MODE_LM>(A, pop<N>(A, P_LM, 0), cta, smem, Ly, bars, tmem, buf, fph, tid);
    tstamp(A, cta, 2 + 7 * A.L, 0, tid);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, kTmemCols);
  if (tid == 0) {  // never leave with a copy still writing shared memory (bounded waits)
    const int gi = issued_s[0], ai = issued_s[1];
    for (int it = gi > nst ? gi - nst : 0; it < gi; ++it)
      if (!mbar_wait(bars + 8u * (it % nst), (it / nst) & 1, A.err, kErrDrain)) break;  // even after an abort
    for (int it = ai > kAStages ? ai - kAStages : 0; it < ai; ++it)
      if (!mbar_wait(abars + 8u * (it % kAStages), (it / kAStages) & 1, A.err, kErrDrain)) break;
  }
}

// ------------------------------------------------------------------ host side
static bool encode_cache_map5(CUtensorMap* m, const void* base, int layers, int batch, int nkv, int64_t cap,
                              int64_t cs_b, int64_t cs_h, int64_t c_ls) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[5] = {(cuuint64_t)kHeadDim, (cuuint64_t)cap, (cuuint64_t)nkv, (cuuint64_t)batch,
                              (cuuint64_t)layers};
  const cuuint64_t strides[4] = {(cuuint64_t)kHeadDim * 2, (cuuint64_t)cs_h * 2, (cuuint64_t)cs_b * 2,
                                 (cuuint64_t)c_ls * 2};
  const cuuint32_t box[5] = {64, (cuuint32_t)kAKeys, 1, 1, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct TcStepPlan {
  int N, grid, nst, smem, asmax;
  int64_t wn[P_KINDS], wk[P_KINDS], total[P_KINDS];
  int smax[P_KINDS];
  int64_t off_counters, off_abort, off_tickets, off_lm_ticket, off_cta_val, off_cta_idx, off_partials, off_aacc,
      off_aml, off_atickets, off_fx_o, off_fx_d, bytes;
};

static int tc_step_plan(const qd_step_desc* d, TcStepPlan* p) {
  if (!d) return set_error(QD_ERR_ARG, "null step descriptor");
  const int64_t L = d->layers, H = d->hidden, I = d->inter, nq = d->nq_heads, nkv = d->nkv_heads, B = d->batch;
  if (L < 1 || H % 128 || I % 64 || (2 * I) % 128 || nq != 4 * nkv || nkv < 1 || nq > 32 || d->vocab < 1 || B < 1 ||
      B > 64 || d->cap < 1)
    return set_error(QD_ERR_UNSUPPORTED, "tc step: unsupported shape (H %% 128, I %% 64, 4 q heads per KV head, "
                                         "head_dim 128, 1 <= batch <= 64)");
  const int N = (int)((B + 15) / 16 * 16);
  p->N = N;
  const int G = host_sm_count();
  p->grid = G;
  const int64_t vocab_rows = (d->vocab + kBlockRows - 1) / kBlockRows * kBlockRows;
  const int64_t n_rows[P_KINDS] = {(nq + 2 * nkv) * 128, H, 2 * I, H, vocab_rows};
  const int64_t ks[P_KINDS] = {H, nq * 128, H, I, H};
  int64_t max_groups = 0, max_partials = 0;
  for (int k = 0; k < P_KINDS; ++k) {
    const int64_t groups = n_rows[k] / kBlockRows;
    const int kblocks = (int)(ks[k] / kBlockCols);
    p->wn[k] = n_rows[k];
    p->wk[k] = ks[k];
    p->total[k] = groups * kblocks;
    if (p->total[k] < G) return set_error(QD_ERR_UNSUPPORTED, "tc step: a projection has fewer blocks than SMs");
    p->smax[k] = stream_k_smax(groups, kblocks, G);
    if (groups > max_groups) max_groups = groups;
    const int64_t part = groups * p->smax[k] * N * kBlockRows * 4;
    if (part > max_partials) max_partials = part;
  }
  const int64_t pairs = B * nkv;
  int64_t ag = G;
  const int64_t per_pair = (d->cap + kAKeys - 1) / kAKeys;
  int64_t asmax = 2 * ((ag + pairs - 1) / pairs) + 2;
  if (asmax > per_pair) asmax = per_pair;
  if (asmax > kAStageMax) return set_error(QD_ERR_UNSUPPORTED, "tc step: too few (sequence, KV head) pairs");
  p->asmax = (int)asmax;
  int nst = 8;
  while (nst > 1 && tc_step_layout(N, nst).total + 1024 > 227 * 1024) --nst;
  if (nst < 2) return set_error(QD_ERR_UNSUPPORTED, "tc step: shared memory too small");
  p->nst = nst;
  p->smem = tc_step_layout(N, nst).total + 1024;
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  p->off_counters = take((2 + 7 * L) * 4);
  p->off_abort = take(4);
  p->off_tickets = take(max_groups * 4);
  p->off_lm_ticket = take(4);
  p->off_cta_val = take((int64_t)N * G * 4);
  p->off_cta_idx = take((int64_t)N * G * 4);
  p->off_partials = take(max_partials);
  p->off_aacc = take(pairs * asmax * kGroup * kHeadDim * 4);
  p->off_aml = take(pairs * asmax * kGroup * 2 * 4);
  p->off_atickets = take(pairs * 4);
  p->off_fx_o = take(B * H * 8);
  p->off_fx_d = take(B * H * 8);
  p->bytes = off;
  return QD_OK;
}

template <int N>
static int launch_tc_step(const TcStepArgs& a, int smem, cudaStream_t stream) {
  auto kern = tc_step_kernel<N>;
  if (int rc = set_max_dynamic_smem((const void*)kern, smem)) return rc;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kPThreads, smem);
  if (e != cudaSuccess || per_sm < 1)
    return set_error(QD_ERR_UNSUPPORTED, "tc step kernel does not fit on an SM (smem %d B)", smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: CTAs wait on one another's results
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[1] = {(void*)&a};
  e = cudaLaunchKernelExC(&cfg, (const void*)kern, args);
  if (e != cudaSuccess) return set_error(QD_ERR_CUDA, "tc step launch: %s", cudaGetErrorString(e));
  return QD_OK;
}

}  // namespace qd

using namespace qd;

extern "C" int qd_tc_decode_step_plan(const qd_step_desc* d, int64_t* scratch_bytes, int* n_pad) {
  TcStepPlan p;
  if (int rc = tc_step_plan(d, &p)) return rc;
  if (scratch_bytes) *scratch_bytes = p.bytes;
  if (n_pad) *n_pad = p.N;
  return QD_OK;
}

extern "C" int qd_tc_decode_step(const qd_step_desc* d, void* xh, void* xa, void* xi, void* scratch,
                                 int64_t scratch_bytes, cudaStream_t stream) {
  TcStepPlan p;
  if (int rc = tc_step_plan(d, &p)) return rc;
  if (!scratch || scratch_bytes < p.bytes)
    return set_error(QD_ERR_SCRATCH, "scratch %lld B < %lld B", (long long)scratch_bytes, (long long)p.bytes);
  const void* ptrs[] = {d->w_qkv, d->w_o, d->w_gu, d->w_down, d->e_packed, d->ln1, d->ln2, d->q_norm, d->k_norm,
                        d->final_norm, d->tok, d->pos, d->x, d->q, d->k_cache, d->v_cache, d->cos, d->sin, d->err,
                        xh, xa, xi};
  for (const void* q : ptrs)
    if (!q) return set_error(QD_ERR_ARG, "tc step: null pointer");
  for (const void* q : {d->w_qkv, d->w_o, d->w_gu, d->w_down, d->e_packed, (const void*)d->x, (const void*)d->q,
                        (const void*)d->k_cache, (const void*)d->v_cache, d->ln1, d->ln2, d->final_norm,
                        (const void*)xh, (const void*)xa, (const void*)xi})
    if (!aligned16(q)) return set_error(QD_ERR_ARG, "tc step: buffers must be 16-byte aligned");
  if (d->cs_h < d->cap * 128 || d->cs_b < d->nkv_heads * d->cs_h || d->cache_layer_stride < d->batch * d->cs_b ||
      d->cs_h % 8 || d->cs_b % 8 || d->cache_layer_stride % 8)
    return set_error(QD_ERR_ARG, "tc step: cache strides");
  if (d->logits && d->ld_logits < d->vocab) return set_error(QD_ERR_ARG, "tc step: ld_logits < vocab");
  const int64_t H = d->hidden, I = d->inter, nq = d->nq_heads, nkv = d->nkv_heads;
  if (d->w_qkv_layer_bytes < (nq + 2 * nkv) * 128 * H * 2 || d->w_o_layer_bytes < H * nq * 128 * 2 ||
      d->w_gu_layer_bytes < 2 * I * H * 2 || d->w_down_layer_bytes < H * I * 2)
    return set_error(QD_ERR_ARG, "tc step: per-layer weight strides smaller than the packed matrices");
  TcStepArgs a = {};
  if (!encode_cache_map5(&a.tk, d->k_cache, (int)d->layers, (int)d->batch, (int)nkv, d->cap, d->cs_b, d->cs_h,
                         d->cache_layer_stride) ||
      !encode_cache_map5(&a.tv, d->v_cache, (int)d->layers, (int)d->batch, (int)nkv, d->cap, d->cs_b, d->cs_h,
                         d->cache_layer_stride))
    return set_error(QD_ERR_CUDA, "cuTensorMapEncodeTiled failed for the KV cache");
  const void* ws[P_KINDS] = {d->w_qkv, d->w_o, d->w_gu, d->w_down, d->e_packed};
  const int64_t wlb[P_KINDS] = {d->w_qkv_layer_bytes, d->w_o_layer_bytes, d->w_gu_layer_bytes, d->w_down_layer_bytes,
                                0};
  for (int k = 0; k < P_KINDS; ++k) {
    a.w[k] = static_cast<const char*>(ws[k]);
    a.wlb[k] = wlb[k];
    a.wn[k] = p.wn[k];
    a.wk[k] = p.wk[k];
    a.total[k] = p.total[k];
    a.smax[k] = p.smax[k];
  }
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
  a.m_act = (int)d->batch;
  a.grid = p.grid;
  a.nst = p.nst;
  a.asmax = p.asmax;
  a.vocab = d->vocab;
  a.eps = (float)d->eps;
  a.scale = (float)d->scale;
  a.tok = d->tok;
  a.pos = d->pos;
  a.x = static_cast<__nv_bfloat16*>(d->x);
  a.q = static_cast<__nv_bfloat16*>(d->q);
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
  a.xh = static_cast<__nv_bfloat16*>(xh);
  a.xa = static_cast<__nv_bfloat16*>(xa);
  a.xi = static_cast<__nv_bfloat16*>(xi);
  a.err = d->err;
  char* sc = static_cast<char*>(scratch);
  a.counters = reinterpret_cast<int*>(sc + p.off_counters);
  a.abort_flag = reinterpret_cast<int*>(sc + p.off_abort);
  a.fx_o = reinterpret_cast<int64_t*>(sc + p.off_fx_o);
  a.fx_d = reinterpret_cast<int64_t*>(sc + p.off_fx_d);
  a.tickets = reinterpret_cast<int*>(sc + p.off_tickets);
  a.lm_ticket = reinterpret_cast<int*>(sc + p.off_lm_ticket);
  a.cta_val = reinterpret_cast<float*>(sc + p.off_cta_val);
  a.cta_idx = reinterpret_cast<int*>(sc + p.off_cta_idx);
  a.partials = reinterpret_cast<float*>(sc + p.off_partials);
  a.apart_acc = reinterpret_cast<float*>(sc + p.off_aacc);
  a.apart_ml = reinterpret_cast<float*>(sc + p.off_aml);
  a.atickets = reinterpret_cast<int*>(sc + p.off_atickets);
  a.trace = d->trace;
  switch (p.N) {
    case 16: return launch_tc_step<16>(a, p.smem, stream);
    case 32: return launch_tc_step<32>(a, p.smem, stream);
    case 48: return launch_tc_step<48>(a, p.smem, stream);
    case 64: return launch_tc_step<64>(a, p.smem, stream);
  }
  return set_error(QD_ERR_UNSUPPORTED, "tc step: batch padding %d", p.N);
}
