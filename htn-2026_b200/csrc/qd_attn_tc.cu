// Tensor-core (tcgen05) GQA flash-decode for large batch x length, sm_100a.
//
// Same work split as the streaming kernel (qd_attn_stream.cu): the 128-key chunks of every (sequence,
// KV head) pair, T = pairs x chunks, dealt out stream-K over the CTAs; a pair split across CTAs is
// merged by its last CTA in CTA order. Per chunk:
//   q.k   S[key, h] = K[key, :] . q[h, :]       one M=128 (keys) x N=16 (4 heads, 12 zero rows) x K=128
//                                                tcgen05.mma chain, K-major operands
//   softmax over the chunk's keys per head in fp32 (one thread per key, scores read from tensor memory),
//         running max / sum, probabilities rounded to BF16 (engine/kernels/decode_attn.py:1-11)
//   P.V   O[d, h] = V[:, d]^T . P[h, :]^T      M=128 (dims) x N=16 x K=128 (keys); V is the MN-major
//                                                operand, P the K-major one
// and the fp32 accumulator of each (dim, head) lives in the thread of that dim: acc = acc * alpha + O.
// K and V move through a 3-stage ring by TMA (4-D tensor maps over the [B, nkv, cap, 128] cache, two
// 64-dim boxes of 128 keys per operand, 128-byte swizzle; a pair's last, partial chunk only as many
// 32-key boxes as hold keys); keys past the cache read as zeros, scores of keys past the valid length
// are masked and those V rows zeroed in shared memory before P.V. Warps 0-3 run softmax and the
// epilogue (tensor-memory lanes 0-127), warp 4 issues the copies, warp 5 issues the MMAs. No
// multicast anywhere.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "qd_attn_dev.cuh"
#include "qd_plan.h"
#include "qd_umma.cuh"

namespace qd {

constexpr int kTKeys = 128;                // keys per chunk (the q.k MMA's M)
constexpr int kTBox = kTKeys * 128;        // one [128 keys][64 dims] BF16 box: 16 KiB
constexpr int kTStage = 4 * kTBox;         // K dims 0-63, K dims 64-127, V dims 0-63, V dims 64-127
constexpr int kTStages = 3;
constexpr int kTTailKeys = 32;             // a pair's last, partial chunk is copied in boxes of 32 keys
constexpr int kTTailBox = kTTailKeys * 128;  // [32 keys][64 dims] BF16: 4 KiB
constexpr int kTN = 16;                    // MMA N: the 4 query heads of the KV head + 12 zero rows
constexpr int kTThreads = 192;
constexpr int kTSO = 3;                    // S / O accumulator sets in tensor memory
constexpr int kTCols = 128;                // tensor memory: S[3] and O[3], 16 columns each (allocated as 128)
constexpr int kTSoftBar = 1;               // named barrier of warps 0-3
constexpr int kTStageMax = 160;            // merge staging: 3 x 4 x smax floats

struct alignas(64) TcAttnArgs {
  CUtensorMap tk, tv;            // boxes of 128 keys
  CUtensorMap tk_tail, tv_tail;  // boxes of kTTailKeys keys
  const __nv_bfloat16* q;
  const int64_t* pos;
  __nv_bfloat16* out;
  int out_npad;  // 0: out [B, nq, 128]; else the O projection's packed operand [nq * 2][out_npad][64]
  int batch, nq, nkv, grid, smax;
  int64_t cap;
  float scale;
  float* part_acc;  // [pairs][smax][4][128]
  float* part_ml;   // [pairs][smax][4][2]
  int* tickets;     // [pairs], chunks arrived
  int* err;
};

struct TcAttnLayout {
  static constexpr int stages = 0;
  static constexpr int qb = kTStages * kTStage;          // [2 dim halves][16 rows][128 B]
  static constexpr int pb = qb + 2 * kTN * 128;          // [2 buffers][2 key halves][16 rows][128 B]
  static constexpr int stg = pb + 2 * 2 * kTN * 128;     // merge staging
  static constexpr int red = stg + 3 * kGroup * kTStageMax * 4;  // [2][4 warps][4 heads] maxima, [4][4] sums
  static constexpr int bars = red + 3 * 4 * kGroup * 4;
  static constexpr int nbars = 2 * kTStages + 3 * kTSO + 2 + 1;  // full, empty, s_full[3], o_full[3], d_free[3],
                                                                 // p_full[2], q_ready
  static constexpr int misc = bars + nbars * 8;           // tmem slot, flag, issued
  static constexpr int total = misc + 16;
};

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar), "l"(policy)
      : "memory");
}

// element index of output (sequence b, query head hq, dim d) in either output layout
__device__ __forceinline__ int64_t attn_out_index(const TcAttnArgs& a, int b, int hq, int d) {
  if (!a.out_npad) return ((int64_t)b * a.nq + hq) * kHeadDim + d;
  const int k = hq * kHeadDim + d, kb = k >> 6, c = k & 63;
  return ((int64_t)kb * a.out_npad + b) * 64 + (((c >> 3) ^ (b & 7)) << 3) + (c & 7);
}

// byte offset of element (row, col) in a [rows][64] BF16 128-byte-swizzled tile (1 KiB-aligned base)
__device__ __forceinline__ uint32_t sw128_off(int row, int col) {
  return (uint32_t)(row * 128 + ((((col >> 3) ^ (row & 7)) & 7) << 4) + ((col & 7) << 1));
}

__global__ void __launch_bounds__(kTThreads, 1) attn_tc_kernel(const __grid_constant__ TcAttnArgs a) {
  extern __shared__ __align__(1024) char smem_raw[];
  char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  using Ly = TcAttnLayout;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;

  // With pdl, q and the new token's K/V (each pair's last chunk) come from the preceding kernel; the
  // position and the keys before it were written before that kernel started (it waited on its own
  // predecessor before letting this grid in). So the set-up and the copies of chunks that are not a
  // pair's last go out before the dependency wait, overlapping the preceding kernel's tail.
  const int64_t len = attn_len_at(ld_cg_s64(a.pos), a.cap, a.err, tid == 0 && cta == 0);
  const int nch = (int)((len + kTKeys - 1) / kTKeys);
  const int pairs = a.batch * a.nkv;
  const int64_t T = (int64_t)pairs * nch;
  const int G = (int)(T < a.grid ? T : a.grid);  // short lengths: the first T CTAs only
  if (cta >= G) return;                          // nothing allocated, issued or armed yet
  const int64_t c_begin = part_begin(T, G, cta), c_end = part_begin(T, G, cta + 1);
  const int n = (int)(c_end - c_begin);

  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + Ly::bars;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (kTStages + s); };
  auto sfull_bar = [&](int b) { return bars + 8u * (2 * kTStages + b); };              // b < kTSO
  auto ofull_bar = [&](int b) { return bars + 8u * (2 * kTStages + kTSO + b); };       // b < kTSO
  auto dfree_bar = [&](int b) { return bars + 8u * (2 * kTStages + 2 * kTSO + b); };   // b < kTSO
  auto pfull_bar = [&](int b) { return bars + 8u * (2 * kTStages + 3 * kTSO + b); };   // b < 2
  const uint32_t qready_bar = bars + 8u * (2 * kTStages + 3 * kTSO + 2);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + Ly::misc);
  int* issued_s = reinterpret_cast<int*>(smem + Ly::misc + 8);

  if (tid == 0) {
    for (int s = 0; s < kTStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < kTSO; ++b) {
      mbar_init(sfull_bar(b), 1);
      mbar_init(ofull_bar(b), 1);
      mbar_init(dfree_bar(b), 4);
    }
    for (int b = 0; b < 2; ++b) mbar_init(pfull_bar(b), 4);
    mbar_init(qready_bar, 4);
    fence_mbar_init();
    *issued_s = 0;
  }
  if (warp == 5) tmem_alloc(smem_u32(tslot), kTCols);
  if (warp < 4) {  // zero the q and P operand tiles (rows 4..15 stay zero: the padded heads)
    for (int i = tid; i < (Ly::stg - Ly::qb) / 16; i += 128)
      *reinterpret_cast<uint4*>(smem + Ly::qb + 16 * i) = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tS0 = tmem, tO0 = tmem + kTSO * kTN;

  if (warp == 4) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int pair = (int)(c_begin / nch), ci = (int)(c_begin - (int64_t)pair * nch);
      int slot = 0, round = 0, issued = 0;
      bool dep_done = false;
      for (int i = 0; i < n; ++i) {
        if (round > 0 && !mbar_wait(empty_bar(slot), (round - 1) & 1, a.err, kErrWaitEmpty)) break;
        if (!dep_done && ci == nch - 1) {  // this chunk holds the row the preceding kernel appends
          grid_dep_wait();
          dep_done = true;
        }
        const int b = pair / a.nkv, kvh = pair - b * a.nkv, k0 = ci * kTKeys;
        const uint32_t st = sbase + Ly::stages + slot * kTStage;
        const int64_t nk = len - k0;
        if (nk >= kTKeys) {
          mbar_arrive_expect_tx(full_bar(slot), kTStage);  // rows past the cache are zero-filled, counted
          tma_load_4d(st, &a.tk, 0, k0, kvh, b, full_bar(slot), pol);
          tma_load_4d(st + kTBox, &a.tk, 64, k0, kvh, b, full_bar(slot), pol);
          tma_load_4d(st + 2 * kTBox, &a.tv, 0, k0, kvh, b, full_bar(slot), pol);
          tma_load_4d(st + 3 * kTBox, &a.tv, 64, k0, kvh, b, full_bar(slot), pol);
        } else {
          // the pair's last chunk: only the 32-key row blocks that hold keys (at 4 KiB steps the
          // 128-byte swizzle pattern is that of the full box); the rows left stale are masked in the
          // softmax (K) and zeroed before P.V (V)
          const int nb = (int)((nk + kTTailKeys - 1) / kTTailKeys);
          mbar_arrive_expect_tx(full_bar(slot), (uint32_t)(4 * nb * kTTailBox));
          for (int j = 0; j < nb; ++j) {
            const uint32_t r = (uint32_t)(j * kTTailBox);
            const int kj = k0 + j * kTTailKeys;
            tma_load_4d(st + r, &a.tk_tail, 0, kj, kvh, b, full_bar(slot), pol);
            tma_load_4d(st + kTBox + r, &a.tk_tail, 64, kj, kvh, b, full_bar(slot), pol);
            tma_load_4d(st + 2 * kTBox + r, &a.tv_tail, 0, kj, kvh, b, full_bar(slot), pol);
            tma_load_4d(st + 3 * kTBox + r, &a.tv_tail, 64, kj, kvh, b, full_bar(slot), pol);
          }
        }
        ++issued;
        if (++ci == nch) {
          ci = 0;
          ++pair;
        }
        if (++slot == kTStages) {
          slot = 0;
          ++round;
        }
      }
      *issued_s = issued;
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id_qk = umma_idesc_bf16(kTN, false), id_pv = umma_idesc_bf16(kTN, true);
      bool ok = mbar_wait(qready_bar, 0, a.err, kErrWaitFull);
      int qph = 1;
      int ci_next = (int)(c_begin % nch);  // chunk-in-pair of the next q.k to issue
      auto issue_qk = [&](int i) {
        const int slot = i % kTStages, b = i % kTSO;
        if (ok) ok = mbar_wait(full_bar(slot), (i / kTStages) & 1, a.err, kErrWaitFull);
        if (ok && i >= kTSO) ok = mbar_wait(dfree_bar(b), ((i / kTSO) - 1) & 1, a.err, kErrWaitFull);
        if (ok && i > 0 && ci_next == 0) {  // first chunk of a new pair: its q must be in place
          ok = mbar_wait(qready_bar, qph & 1, a.err, kErrWaitFull);
          ++qph;
        }
        tc_fence_after();
        if (ok) {
          const uint32_t st = sbase + Ly::stages + slot * kTStage;
#pragma unroll
          for (int j = 0; j < 8; ++j)  // 16 dims per MMA: +32 B inside a 64-dim box, the next box after 4
            umma_bf16(tS0 + b * kTN, umma_desc_sw128(st + (j >> 2) * kTBox + (j & 3) * 32),
                      umma_desc_sw128(sbase + Ly::qb + (j >> 2) * (kTN * 128) + (j & 3) * 32), id_qk,
                      j > 0 ? 1u : 0u);
        }
        umma_commit(sfull_bar(b));
        if (++ci_next == nch) ci_next = 0;
      };
      if (n > 0) issue_qk(0);
      for (int i = 0; i < n; ++i) {
        // the next chunk's q.k goes first unless it starts a new pair: then it waits for that pair's q,
        // and this chunk's P.V must not wait with it
        const bool next_new_pair = (i + 1 < n) && ci_next == 0;
        if (i + 1 < n && !next_new_pair) issue_qk(i + 1);
        const int slot = i % kTStages, b = i & 1, bo = i % kTSO;
        if (ok) ok = mbar_wait(pfull_bar(b), (i >> 1) & 1, a.err, kErrWaitFull);
        tc_fence_after();
        if (ok) {
          const uint32_t vst = sbase + Ly::stages + slot * kTStage + 2 * kTBox;
#pragma unroll
          for (int j = 0; j < 8; ++j)  // 16 keys per MMA: two 8-key atoms of 1 KiB; dims 64-127 one box on
            umma_bf16(tO0 + bo * kTN, umma_desc_sw128(vst + j * 2048, kTBox, 1024),
                      umma_desc_sw128(sbase + Ly::pb + b * (2 * kTN * 128) + (j >> 2) * (kTN * 128) + (j & 3) * 32),
                      id_pv, j > 0 ? 1u : 0u);
        }
        umma_commit(ofull_bar(bo));
        umma_commit(empty_bar(slot));
        if (next_new_pair) issue_qk(i + 1);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax + epilogue (warps 0-3)
    float* red = reinterpret_cast<float*>(smem + Ly::red);
    int pair = (int)(c_begin / nch), ci = (int)(c_begin - (int64_t)pair * nch);
    int seg_first = ci;
    float m_run[kGroup], l_thr[kGroup], acc[kGroup];
    // q of a pair: loaded into registers one pair ahead (its latency hides behind the current pair),
    // stored into the operand tile when the previous pair's last q.k is done
    const int pair_last = (int)((c_end - 1) / nch);
    unsigned short qn[kGroup];
    auto load_q = [&](int pr) {
      const int b = pr / a.nkv, kvh = pr - b * a.nkv;
#pragma unroll
      for (int h = 0; h < kGroup; ++h)
        qn[h] = __ldcg(reinterpret_cast<const unsigned short*>(a.q) + ((int64_t)b * a.nq + kvh * kGroup + h) * kHeadDim +
                       tid);
    };
    auto put_q = [&](int pr) {  // store the loaded q of pair pr, then load the following pair's
#pragma unroll
      for (int h = 0; h < kGroup; ++h)
        *reinterpret_cast<unsigned short*>(smem + Ly::qb + (tid >> 6) * (kTN * 128) + sw128_off(h, tid & 63)) = qn[h];
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(qready_bar);
      if (pr + 1 <= pair_last) load_q(pr + 1);
    };
    grid_dep_wait();  // q comes from the preceding kernel
    grid_dep_launch();
    load_q(pair);
    auto reset_state = [&]() {
#pragma unroll
      for (int h = 0; h < kGroup; ++h) {
        m_run[h] = -INFINITY;
        l_thr[h] = 0.f;
        acc[h] = 0.f;
      }
    };
    put_q(pair);
    reset_state();
    bool ok = true;
    // O of chunk j: thread tid holds dim tid of the 4 heads; acc = acc * alpha_j + O_j
    auto consume_o = [&](int j, const float* al) {
      const int bo = j % kTSO;
      if (ok) ok = mbar_wait(ofull_bar(bo), (j / kTSO) & 1, a.err, kErrWaitFull);
      tc_fence_after();
      float o[4];
      tmem_ld4(tO0 + bo * kTN + ((uint32_t)(32 * warp) << 16), o);
      tmem_wait_ld();
#pragma unroll
      for (int h = 0; h < kGroup; ++h) acc[h] = fmaf(acc[h], al[h], o[h]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dfree_bar(bo));
    };
    bool have_pend = false;
    float pend_alpha[kGroup];
    for (int i = 0; i < n; ++i) {
      const int slot = i % kTStages, b = i & 1, bs = i % kTSO;
      const int k0 = ci * kTKeys;
      const int nk = (int)((len - k0) < kTKeys ? (len - k0) : kTKeys);
      if (ok) ok = mbar_wait(sfull_bar(bs), (i / kTSO) & 1, a.err, kErrWaitFull);
      tc_fence_after();
      float s[4];
      tmem_ld4(tS0 + bs * kTN + ((uint32_t)(32 * warp) << 16), s);
      tmem_wait_ld();
      const bool valid = tid < nk;
      float mx[kGroup];
#pragma unroll
      for (int h = 0; h < kGroup; ++h) {
        s[h] = valid ? s[h] * a.scale : -INFINITY;
        mx[h] = warp_max(s[h]);
      }
      float* rb = red + (i & 1) * 16;
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < kGroup; ++h) rb[warp * 4 + h] = mx[h];
      }
      named_bar(kTSoftBar, 128);
      float alpha[kGroup];
#pragma unroll
      for (int h = 0; h < kGroup; ++h) {
        const float mc = fmaxf(fmaxf(rb[h], rb[4 + h]), fmaxf(rb[8 + h], rb[12 + h]));
        const float m_new = fmaxf(m_run[h], mc);
        alpha[h] = expf(m_run[h] - m_new);  // exp(-inf) = 0 on a segment's first chunk
        const float p = valid ? expf(s[h] - m_new) : 0.f;
        l_thr[h] = l_thr[h] * alpha[h] + p;
        m_run[h] = m_new;
        *reinterpret_cast<__nv_bfloat16*>(smem + Ly::pb + b * (2 * kTN * 128) + (tid >> 6) * (kTN * 128) +
                                          sw128_off(h, tid & 63)) = __float2bfloat16_rn(p);
      }
      if (nk < kTKeys) {  // V rows past the valid length may hold anything: zero them for P.V
        char* vst = smem + Ly::stages + slot * kTStage + 2 * kTBox;
        for (int r = nk + tid; r < kTKeys; r += 128)
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4*>(vst + r * 128 + 16 * c) = make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(vst + kTBox + r * 128 + 16 * c) = make_uint4(0u, 0u, 0u, 0u);
          }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(pfull_bar(b));
      const bool pair_end = (ci == nch - 1) || (i == n - 1);
      // the next chunk starts a new pair: its q goes in now, so its q.k can run during this P.V
      if (pair_end && i + 1 < n) put_q(pair + 1);
      // O of the previous chunk of this segment (deferred by one chunk, so its P.V runs during this
      // chunk's softmax), then this chunk's own O only where the segment ends
      if (have_pend) {
        consume_o(i - 1, pend_alpha);
        have_pend = false;
      }
      if (!pair_end) {
#pragma unroll
        for (int h = 0; h < kGroup; ++h) pend_alpha[h] = alpha[h];
        have_pend = true;
        ++ci;
      } else {
        consume_o(i, alpha);
        // ---- flush the pair segment [seg_first, ci]: sums over the 128 key threads, then out or partial
        float l[kGroup];
#pragma unroll
        for (int h = 0; h < kGroup; ++h) l[h] = warp_sum(l_thr[h]);
        float* lb = red + 32;
        if (lane == 0) {
#pragma unroll
          for (int h = 0; h < kGroup; ++h) lb[warp * 4 + h] = l[h];
        }
        named_bar(kTSoftBar, 128);
#pragma unroll
        for (int h = 0; h < kGroup; ++h) l[h] = ((lb[h] + lb[4 + h]) + lb[8 + h]) + lb[12 + h];
        const int bb = pair / a.nkv, kvh = pair - bb * a.nkv;
        if (seg_first == 0 && ci == nch - 1) {
#pragma unroll
          for (int h = 0; h < kGroup; ++h)
            a.out[attn_out_index(a, bb, kvh * kGroup + h, tid)] = __float2bfloat16_rn(acc[h] / l[h]);
        } else {
          const int64_t gc0 = (int64_t)pair * nch;
          const int c_lo = part_owner(T, G, gc0);
          const int pslot = cta - c_lo;
          const int nseg = part_owner(T, G, gc0 + nch - 1) - c_lo + 1;
          if (pslot < 0 || pslot >= a.smax || nseg > a.smax) {  // cannot happen with the plan's smax
            if (tid == 0 && a.err) atomicOr(a.err, kErrDep);
          } else {
            const int64_t prow = ((int64_t)pair * a.smax + pslot) * kGroup;
#pragma unroll
            for (int h = 0; h < kGroup; ++h) __stcg(a.part_acc + (prow + h) * kHeadDim + tid, acc[h]);
            if (tid < 2 * kGroup) __stcg(a.part_ml + prow * 2 + tid, (tid & 1) ? l[tid >> 1] : m_run[tid >> 1]);
            named_bar(kTSoftBar, 128);
            int* flag = reinterpret_cast<int*>(smem + Ly::misc + 4);
            if (tid == 0) {
              const int cnt = ci - seg_first + 1;
              *flag = (atom_add_acq_rel(a.tickets + pair, cnt) + cnt == nch) ? 1 : 0;
            }
            named_bar(kTSoftBar, 128);
            if (*flag) {
              float* mm = reinterpret_cast<float*>(smem + Ly::stg);
              float* ll = mm + kGroup * nseg;
              float* ww = ll + kGroup * nseg;
              const int64_t prow0 = (int64_t)pair * a.smax * kGroup;
              for (int t = tid; t < kGroup * nseg; t += 128) {
                const int h = t / nseg, sg = t - h * nseg;
                mm[t] = ld_cg_f32(a.part_ml + (prow0 + (int64_t)sg * kGroup + h) * 2);
                ll[t] = ld_cg_f32(a.part_ml + (prow0 + (int64_t)sg * kGroup + h) * 2 + 1);
              }
              named_bar(kTSoftBar, 128);
              for (int t = tid; t < kGroup * nseg; t += 128) {
                const int h = t / nseg;
                float m2 = -INFINITY;
                for (int sg = 0; sg < nseg; ++sg) m2 = fmaxf(m2, mm[h * nseg + sg]);
                ww[t] = (mm[t] == -INFINITY) ? 0.f : expf(mm[t] - m2);
              }
              named_bar(kTSoftBar, 128);
#pragma unroll
              for (int h = 0; h < kGroup; ++h) {
                float nm = 0.f;
                for (int s0 = 0; s0 < nseg; s0 += 8) {
                  float av[8];
#pragma unroll
                  for (int j = 0; j < 8; ++j)
                    av[j] = (s0 + j < nseg)
                                ? ld_cg_f32(a.part_acc + (prow0 + (int64_t)(s0 + j) * kGroup + h) * kHeadDim + tid)
                                : 0.f;
#pragma unroll
                  for (int j = 0; j < 8; ++j)
                    if (s0 + j < nseg) nm = fmaf(av[j], ww[h * nseg + s0 + j], nm);
                }
                float den = 0.f;
                for (int sg = 0; sg < nseg; ++sg) den = fmaf(ll[h * nseg + sg], ww[h * nseg + sg], den);
                a.out[attn_out_index(a, bb, kvh * kGroup + h, tid)] = __float2bfloat16_rn(nm / den);
              }
              if (tid == 0) atomicExch(a.tickets + pair, 0);
            }
          }
        }
        named_bar(kTSoftBar, 128);  // staging and the sum buffer are reused
        if (++ci == nch) {
          ci = 0;
          ++pair;
        }
        seg_first = ci;
        reset_state();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, kTCols);
  if (tid == 0) {  // never leave with a copy still writing shared memory (bounded waits)
    const int issued = *issued_s;
    for (int it = issued > kTStages ? issued - kTStages : 0; it < issued; ++it)
      if (!mbar_wait(full_bar(it % kTStages), (it / kTStages) & 1, a.err, kErrDrain)) break;
  }
}

static int tc_attn_grid(int pairs, int64_t cap, int grid_hint, int* smax_out) {
  const int64_t max_chunks = (int64_t)pairs * ((cap + kTKeys - 1) / kTKeys);
  int64_t g = grid_hint > 0 ? grid_hint : host_sm_count();
  if (g > (int64_t)79 * pairs) g = (int64_t)79 * pairs;  // smax <= 160
  if (g > max_chunks) g = max_chunks;
  if (g < 1) g = 1;
  int64_t smax = 2 * ((g + pairs - 1) / pairs) + 2;
  const int64_t per_pair = (cap + kTKeys - 1) / kTKeys;
  if (smax > per_pair) smax = per_pair;
  *smax_out = (int)smax;
  return (int)g;
}

static int64_t tc_attn_scratch(int pairs, int smax, int64_t* off_ml, int64_t* off_t) {
  const int64_t rows = (int64_t)pairs * smax * kGroup;
  const int64_t acc = (rows * kHeadDim * 4 + 255) / 256 * 256, ml = (rows * 2 * 4 + 255) / 256 * 256;
  *off_ml = acc;
  *off_t = acc + ml;
  return acc + ml + ((int64_t)pairs * 4 + 255) / 256 * 256;
}

static bool encode_cache_map(CUtensorMap* m, const void* base, int batch, int nkv, int64_t cap, int64_t cs_b,
                             int64_t cs_h, int box_keys) {
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)kHeadDim, (cuuint64_t)cap, (cuuint64_t)nkv, (cuuint64_t)batch};
  const cuuint64_t strides[3] = {(cuuint64_t)kHeadDim * 2, (cuuint64_t)cs_h * 2, (cuuint64_t)cs_b * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_keys, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                                            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace qd

using namespace qd;

extern "C" int qd_attn_tc_plan(int batch, int nkv_heads, int64_t cap, int grid_hint, int* grid, int* smax,
                               int64_t* scratch_bytes) {
  if (batch < 1 || nkv_heads < 1 || cap < 1 || (int64_t)batch * nkv_heads > (1 << 24))
    return set_error(QD_ERR_ARG, "attn tc plan: bad sizes");
  int sm_ = 0;
  const int g = tc_attn_grid(batch * nkv_heads, cap, grid_hint, &sm_);
  int64_t om, ot;
  if (grid) *grid = g;
  if (smax) *smax = sm_;
  if (scratch_bytes) *scratch_bytes = tc_attn_scratch(batch * nkv_heads, sm_, &om, &ot);
  return QD_OK;
}

extern "C" int qd_attn_decode_tc(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos,
                                 void* out, int out_npad, int batch, int nq_heads, int nkv_heads, int64_t cap, int64_t cs_b,
                                 int64_t cs_h, int grid, int smax, float scale, void* scratch, int64_t scratch_bytes,
                                 int* err, int pdl, cudaStream_t stream) {
  if (!q || !k_cache || !v_cache || !pos || !out || !scratch) return set_error(QD_ERR_ARG, "null pointer");
  if (nkv_heads < 1 || nq_heads != nkv_heads * kGroup)
    return set_error(QD_ERR_UNSUPPORTED, "attention is built for %d query heads per KV head", kGroup);
  if (batch < 1 || cap < 1 || (int64_t)batch * nkv_heads > (1 << 24)) return set_error(QD_ERR_ARG, "bad sizes");
  if (out_npad && (out_npad < batch || out_npad % 16 || out_npad > 64 || !aligned16(out)))
    return set_error(QD_ERR_ARG, "out_npad must be 0 or a multiple of 16 in [batch, 64], out 16-byte aligned");
  int want_smax = 0;
  const int want_grid = tc_attn_grid(batch * nkv_heads, cap, grid, &want_smax);
  if (grid != want_grid || smax != want_smax)
    return set_error(QD_ERR_ARG, "grid/smax do not match qd_attn_tc_plan (%d, %d)", want_grid, want_smax);
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || cs_h < cap * kHeadDim ||
      cs_b < (int64_t)nkv_heads * cs_h || cs_h % 8 || cs_b % 8)
    return set_error(QD_ERR_ARG, "cache strides/alignment");
  int64_t om, ot;
  const int64_t need = tc_attn_scratch(batch * nkv_heads, smax, &om, &ot);
  if (scratch_bytes < need)
    return set_error(QD_ERR_SCRATCH, "scratch %lld B < %lld B", (long long)scratch_bytes, (long long)need);
  TcAttnArgs a = {};
  if (!encode_cache_map(&a.tk, k_cache, batch, nkv_heads, cap, cs_b, cs_h, kTKeys) ||
      !encode_cache_map(&a.tv, v_cache, batch, nkv_heads, cap, cs_b, cs_h, kTKeys) ||
      !encode_cache_map(&a.tk_tail, k_cache, batch, nkv_heads, cap, cs_b, cs_h, kTTailKeys) ||
      !encode_cache_map(&a.tv_tail, v_cache, batch, nkv_heads, cap, cs_b, cs_h, kTTailKeys))
    return set_error(QD_ERR_CUDA, "cuTensorMapEncodeTiled failed for the KV cache");
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.pos = pos;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_npad = out_npad;
  a.batch = batch;
  a.nq = nq_heads;
  a.nkv = nkv_heads;
  a.grid = grid;
  a.smax = smax;
  a.cap = cap;
  a.scale = scale;
  char* sc = static_cast<char*>(scratch);
  a.part_acc = reinterpret_cast<float*>(sc);
  a.part_ml = reinterpret_cast<float*>(sc + om);
  a.tickets = reinterpret_cast<int*>(sc + ot);
  a.err = err;
  const int smem = TcAttnLayout::total + 1024;  // + base alignment slack
  if (int rc = set_max_dynamic_smem((const void*)attn_tc_kernel, smem)) return rc;
  return launch_kernel((const void*)attn_tc_kernel, dim3(grid), dim3(kTThreads), smem, pdl, stream, &a);
}
