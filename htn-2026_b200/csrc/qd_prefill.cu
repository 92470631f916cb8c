// Prompt (prefill) kernels for sm_100a: a tcgen05 GEMM over the packed weights, the row RMSNorm and the
// per-head q/k RMSNorm + RoPE + KV-cache write of the prompt positions.
//
// The prefill forward (engine/engine.py:550-592) runs every prompt token through the layers at once,
// so its projections are real GEMMs (rows = tokens). qd_tc_gemm computes
//     out[t, :] = epilogue(x[t, :] . W^T)
// with x [m, k] row-major BF16 and W in the packed 16 KiB-block layout the decode kernels stream, so one
// copy of the weights serves both phases. Tiles are 128 tokens x BN weight rows (BN = 128 or 256):
// A = the token tile, loaded by a 2-D TMA tensor map with the 128-byte swizzle (box 64 columns x 128
// rows, rows past m read as zero); B = BN/128 packed blocks, one bulk copy each - the packed block
// already is a K-major 128-byte-swizzled operand, and two consecutive blocks form one 256-row operand
// (8-row atoms 1 KiB apart). Per 64-column K step: 4 tcgen05.mma (M = 128, N = BN, K = 16) into an
// fp32 accumulator in tensor memory, two accumulators alternating so the epilogue of one tile
// overlaps the MMAs of the next.
//
// Warp roles (192 threads): warps 0-3 epilogue (warp w reads TMEM lanes 32w.., i.e. tokens 32w..),
// warp 4 producer, warp 5 MMA issuer. The CTAs are persistent over the tiles; tiles run in groups of
// kGroupM token tiles x all weight tiles so a group's activations stay in L2 while the weights stream.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "qd_common.cuh"
#include "qd_host.h"
#include "qd_plan.h"
#include "qd_umma.cuh"

namespace qd {

constexpr int kGemmThreads = 192;
constexpr int kGemmEpiWarps = 4;
constexpr int kGroupM = 8;  // token tiles per raster group

enum { GEMM_STORE = 0, GEMM_RES = 1, GEMM_SWIGLU = 2 };

struct alignas(64) GemmArgs {
  CUtensorMap tx;  // x [m, k] BF16, box {64, 128}, 128-byte swizzle
  const char* w;   // packed [ngroups * 128, k]
  __nv_bfloat16* out;
  const __nv_bfloat16* res;
  int64_t ldo, ldr, m, n;
  int kblocks, ngroups, m_tiles, n_tiles, tiles, nst;
  // work units: tiles [0, full_tiles) whole (unit u = tile u), then every later tile in ksplit K-ranges
  // (unit full_tiles + j * ksplit + s = split s of tile full_tiles + j)
  int full_tiles, ksplit, units;
  float* partials;  // [tiles - full_tiles][ksplit][128][BN] fp32 accumulator partials of the split tiles
  int* err;
};

// unit u -> tile t, split s (-1: the whole tile) and its K-block range [kb0, kb1)
__device__ __forceinline__ void gemm_unit(const GemmArgs& a, int u, int* t, int* s, int* kb0, int* kb1) {
  if (u < a.full_tiles) {
    *t = u;
    *s = -1;
    *kb0 = 0;
    *kb1 = a.kblocks;
    return;
  }
  const int v = u - a.full_tiles, j = v / a.ksplit, sp = v - j * a.ksplit;
  *t = a.full_tiles + j;
  *s = sp;
  *kb0 = (int)((int64_t)sp * a.kblocks / a.ksplit);
  *kb1 = (int)((int64_t)(sp + 1) * a.kblocks / a.ksplit);
}

template <int BN>
struct GemmLayout {
  static constexpr int stage = kBlockBytes + BN * 128;  // token tile + BN/128 weight blocks
  static __host__ __device__ int bars(int nst) { return nst * stage; }
  static __host__ __device__ int total(int nst) { return bars(nst) + (2 * nst + 4) * 8 + 16; }
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// tile index -> (token tile, weight tile): groups of kGroupM token tiles, weight tiles outer within
// a group
__device__ __forceinline__ void gemm_tile(int m_tiles, int n_tiles, int t, int* mt, int* nt) {
  const int per_group = kGroupM * n_tiles;
  const int grp = t / per_group, rem = t - grp * per_group;
  const int m0 = grp * kGroupM;
  const int gm = (m_tiles - m0) < kGroupM ? (m_tiles - m0) : kGroupM;
  *mt = m0 + rem % gm;
  *nt = rem / gm;
}

__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1) tc_gemm_kernel(const __grid_constant__ GemmArgs a) {
  extern __shared__ __align__(1024) char smem_raw[];
  char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  using Ly = GemmLayout<BN>;
  const int nst = a.nst;
  const uint32_t ring = smem_u32(smem);
  const uint32_t bars = smem_u32(smem + Ly::bars(nst));
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (nst + s); };
  auto accf_bar = [&](int i) { return bars + 8u * (2 * nst + i); };
  auto acce_bar = [&](int i) { return bars + 8u * (2 * nst + 2 + i); };
  int* misc = reinterpret_cast<int*>(smem + Ly::bars(nst) + (2 * nst + 4) * 8);  // tmem slot, abort, issued
  constexpr uint32_t kCols = 2 * BN;  // two accumulators

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x, G = gridDim.x;
  // programmatic dependent launch both ways. Before griddepcontrol.wait this grid touches no activation
  // and holds no tensor memory (a co-resident CTA of the previous grid may still need to allocate some):
  // it initialises its barriers and the producer prefetches its first weight blocks (never written by
  // the prompt forward) into L2. The next kernel is let in only once the tensor memory is held.
  if (tid == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(accf_bar(i), 1);
      mbar_init(acce_bar(i), kGemmEpiWarps);
    }
    fence_mbar_init();
    misc[1] = 0;
    misc[2] = 0;
  }
  if (warp == 4 && lane == 0 && cta < a.units) {
    // the first unit's weight blocks into L2 (up to 256 KiB) while the previous kernel runs
    int t, sp, mt, nt, kb0, kb1;
    gemm_unit(a, cta, &t, &sp, &kb0, &kb1);
    gemm_tile(a.m_tiles, a.n_tiles, t, &mt, &nt);
    const int nkb = (kb1 - kb0) < 16 / (BN / 128) ? (kb1 - kb0) : 16 / (BN / 128);
    for (int h = 0; h < BN / 128; ++h) {
      const int g = nt * (BN / 128) + h;
      if (g < a.ngroups)
        prefetch_l2(a.w + ((int64_t)g * a.kblocks + kb0) * kBlockBytes, (uint32_t)(nkb * kBlockBytes));
    }
  }
  grid_dep_wait();
  if (warp == 5) tmem_alloc(smem_u32(misc), kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_launch();
  const uint32_t tmem = (uint32_t)misc[0];
  int* abort = misc + 1;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_normal();
      int slot = 0, round = 0, issued = 0;
      bool ok = true;
      for (int u = cta; u < a.units && ok; u += G) {
        int t, sp, mt, nt, kb0, kb1;
        gemm_unit(a, u, &t, &sp, &kb0, &kb1);
        gemm_tile(a.m_tiles, a.n_tiles, t, &mt, &nt);
        const int g0 = nt * (BN / 128);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (round > 0 && !mbar_wait_abort(empty_bar(slot), (round - 1) & 1, a.err, kErrWaitEmpty, abort)) {
            ok = false;
            break;
          }
          const uint32_t st = ring + slot * Ly::stage;
          mbar_arrive_expect_tx(full_bar(slot), (uint32_t)Ly::stage);
          tma_load_2d(st, &a.tx, kb * 64, mt * 128, full_bar(slot), pol);
#pragma unroll
          for (int h = 0; h < BN / 128; ++h) {
            // a missing last group (odd group count) repeats the previous one: computed, never stored
            const int g = (g0 + h < a.ngroups) ? g0 + h : a.ngroups - 1;
            bulk_g2s(st + kBlockBytes * (1 + h), a.w + ((int64_t)g * a.kblocks + kb) * kBlockBytes, kBlockBytes,
                     full_bar(slot), pol);
          }
          ++issued;
          if (++slot == nst) {
            slot = 0;
            ++round;
          }
        }
      }
      misc[2] = issued;
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(BN);
      int slot = 0, fph = 0, i = 0;
      bool ok = true;
      for (int u = cta; u < a.units && ok; u += G, ++i) {
        const int buf = i & 1;
        if (i >= 2 && !mbar_wait_abort(acce_bar(buf), ((i >> 1) - 1) & 1, a.err, kErrWaitFull, abort)) break;
        tc_fence_after();
        int t, sp, kb0, kb1;
        gemm_unit(a, u, &t, &sp, &kb0, &kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_abort(full_bar(slot), fph, a.err, kErrWaitFull, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = ring + slot * Ly::stage, sb = sa + kBlockBytes;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            umma_bf16(tmem + buf * BN, umma_desc_sw128(sa + 32 * j), umma_desc_sw128(sb + 32 * j), idesc,
                      (kb > kb0 || j) ? 1u : 0u);
          umma_commit(empty_bar(slot));
          if (++slot == nst) {
            slot = 0;
            fph ^= 1;
          }
        }
        if (ok) umma_commit(accf_bar(buf));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue: thread = token row
    int i = 0;
    for (int u = cta; u < a.units; u += G, ++i) {
      const int buf = i & 1;
      if (!mbar_wait_abort(accf_bar(buf), (i >> 1) & 1, a.err, kErrWaitFull, abort)) break;
      tc_fence_after();
      int t, sp, kb0, kb1, mt, nt;
      gemm_unit(a, u, &t, &sp, &kb0, &kb1);
      gemm_tile(a.m_tiles, a.n_tiles, t, &mt, &nt);
      const int64_t row = (int64_t)mt * 128 + 32 * warp + lane;
      const bool live = row < a.m;
      const uint32_t tb = tmem + ((uint32_t)(32 * warp) << 16) + buf * BN;
      if (sp >= 0) {
        // split-K: this split's fp32 accumulator rows go to the partials (live rows only); the sum over
        // the splits and the epilogue run in gemm_splitk_sum_kernel
        float* prow =
            a.partials + (((int64_t)(t - a.full_tiles) * a.ksplit + sp) * 128 + 32 * warp + lane) * BN;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tmem_ld32(tb + c, v);
          if (!live) continue;
          float4* d4 = reinterpret_cast<float4*>(prow + c);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            __stcg(d4 + q, make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                       __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3])));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce_bar(buf));
        continue;
      }
      if constexpr (EPI == GEMM_SWIGLU) {
        // group g of the interleaved gate/up matrix: 64 gate rows, then the 64 up rows of the same
        // outputs 64g..64g+63
#pragma unroll 1
        for (int h = 0; h < BN / 128; ++h) {
          const int g = nt * (BN / 128) + h;
          if (g >= a.ngroups) break;
#pragma unroll 1
          for (int j0 = 0; j0 < 64; j0 += 16) {
            uint32_t gr[16], ur[16];
            tmem_ld16_raw(tb + h * 128 + j0, gr);
            tmem_ld16_raw(tb + h * 128 + 64 + j0, ur);
            tmem_wait_ld16(gr);
            tmem_wait_ld16(ur);
            uint32_t o[8];
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              float r2[2];
#pragma unroll
              for (int d = 0; d < 2; ++d) {
                const float gv = bf16r(__uint_as_float(gr[e + d]));
                const float uv = bf16r(__uint_as_float(ur[e + d]));
                const float s = bf16r(gv / (1.0f + expf(-gv)));
                r2[d] = s * uv;
              }
              o[e >> 1] = pack_bf2(r2[0], r2[1]);
            }
            if (live) {
              uint4* dst = reinterpret_cast<uint4*>(a.out + row * a.ldo + (int64_t)g * 64 + j0);
              dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
              dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          const int64_t col = (int64_t)nt * BN + c;  // n % 128 == 0: a 32-column chunk is all in or all out
          uint32_t r0[16], r1[16];
          tmem_ld16_raw(tb + c, r0);
          tmem_ld16_raw(tb + c + 16, r1);
          tmem_wait_ld16(r0);
          tmem_wait_ld16(r1);
          if (!live || col >= a.n) continue;
          float v[32];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            v[e] = bf16r(__uint_as_float(r0[e]));
            v[16 + e] = bf16r(__uint_as_float(r1[e]));
          }
          if constexpr (EPI == GEMM_RES) {
            const uint4* rp = reinterpret_cast<const uint4*>(a.res + row * a.ldr + col);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 u = rp[q];
              const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                v[8 * q + 2 * e] += bf_lo(w4[e]);
                v[8 * q + 2 * e + 1] += bf_hi(w4[e]);
              }
            }
          }
          uint4* dst = reinterpret_cast<uint4*>(a.out + row * a.ldo + col);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_bf2(v[8 * q], v[8 * q + 1]), pack_bf2(v[8 * q + 2], v[8 * q + 3]),
                                pack_bf2(v[8 * q + 4], v[8 * q + 5]), pack_bf2(v[8 * q + 6], v[8 * q + 7]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar(buf));
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, kCols);
  if (tid == 0) {  // no bulk copy may still be writing shared memory when the CTA exits
    const int issued = misc[2];
    for (int it = issued > nst ? issued - nst : 0; it < issued; ++it)
      if (!mbar_wait(full_bar(it % nst), (it / nst) & 1, a.err, kErrDrain)) break;
  }
}

// ------------------------------------------------------------------ row RMSNorm
struct RmsArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* w;
  __nv_bfloat16* out;
  int64_t ldx, ldo, k;
  float eps;
};

// One CTA of 256 threads per row: out = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))) (Qwen3RMSNorm's
// cast placement, engine/engine.py:505-509).
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const __grid_constant__ RmsArgs a) {
  grid_dep_wait();  // launched as a programmatic dependent of the previous prompt kernel
  grid_dep_launch();
  __shared__ float wsum[8];
  const int64_t m = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k8 = (int)(a.k >> 3);
  const __nv_bfloat16* xr = a.x + m * a.ldx;
  float sq = 0.f;
  for (int q = tid; q < k8; q += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + q * 8);
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
  __syncthreads();
  float ss = 0.f;
#pragma unroll
  for (int w8 = 0; w8 < 8; ++w8) ss += wsum[w8];
  const float rstd = 1.0f / sqrtf(ss / (float)a.k + a.eps);
  for (int q = tid; q < k8; q += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + q * 8);
    const uint4 wv = *reinterpret_cast<const uint4*>(a.w + q * 8);
    const uint32_t xu[4] = {v.x, v.y, v.z, v.w};
    const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = bf16r(bf_lo(wu[e]) * bf16r(bf_lo(xu[e]) * rstd));
      const float hi = bf16r(bf_hi(wu[e]) * bf16r(bf_hi(xu[e]) * rstd));
      o[e] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
    }
    *reinterpret_cast<uint4*>(a.out + m * a.ldo + q * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ------------------------------------------------------------------ row argmax (the prompt's first token)
struct ArgmaxArgs {
  const __nv_bfloat16* logits;  // [rows, ld]
  int64_t* out;                 // [rows]
  int64_t ld, n;                // n = entries per row that compete (the vocabulary)
};

// The better of two (value, index) candidates: the larger value, the lower index on an exact tie.
__device__ __forceinline__ bool argmax_better(float v, int64_t i, float bv, int64_t bi) {
  return v > bv || (v == bv && i < bi);
}

// One CTA of 256 threads per row: out[row] = the index of the row's largest BF16 logit, the lowest
// index among exact ties (the greedy rule the reference applies to the prompt's last-position logits,
// engine/engine.py:583-591). 16-byte loads over the row, a scalar tail past the last full vector,
// then a butterfly across each warp and one pass over the 8 warp winners.
__global__ void __launch_bounds__(256) argmax_rows_kernel(const __grid_constant__ ArgmaxArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ float wv[8];
  __shared__ int64_t wi[8];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const __nv_bfloat16* r = a.logits + row * a.ld;
  float best = -INFINITY;
  int64_t bidx = INT64_MAX;
  const int64_t n8 = a.n >> 3;
  for (int64_t q = tid; q < n8; q += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(r + q * 8);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = bf_lo(u[e]), hi = bf_hi(u[e]);
      const int64_t i = q * 8 + 2 * e;
      if (argmax_better(lo, i, best, bidx)) best = lo, bidx = i;
      if (argmax_better(hi, i + 1, best, bidx)) best = hi, bidx = i + 1;
    }
  }
  for (int64_t i = n8 * 8 + tid; i < a.n; i += 256) {
    const float v = __bfloat162float(r[i]);
    if (argmax_better(v, i, best, bidx)) best = v, bidx = i;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t i = __shfl_xor_sync(0xffffffffu, bidx, o);
    if (argmax_better(v, i, best, bidx)) best = v, bidx = i;
  }
  if (lane == 0) wv[warp] = best, wi[warp] = bidx;
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < 8; ++w)
      if (argmax_better(wv[w], wi[w], best, bidx)) best = wv[w], bidx = wi[w];
    a.out[row] = bidx == INT64_MAX ? 0 : bidx;  // a row of NaN only: index 0
  }
}

// ------------------------------------------------------------------ prompt q/k norm + RoPE + cache write
struct QkRopeArgs {
  const __nv_bfloat16* qkv;  // [b * S, (nq + 2 nkv) * 128], token t = i * S + s
  const __nv_bfloat16 *qn, *kn, *cos, *sin;
  __nv_bfloat16* q_out;  // [b * S, nq * 128]
  __nv_bfloat16 *k_cache, *v_cache;
  int64_t ldqkv, ldq, S, cs_b, cs_h, tokens;
  int64_t pos0;  // position of the first token of every sequence (token i * S + s sits at pos0 + s)
  const int32_t* rope_pos;  // optional, per token: the RoPE position (the cache slot stays pos0 + s)
  const int32_t* slot0;     // optional, per sequence: its first token's cache slot, in place of pos0
  int64_t cap;
  int* err;
  int nq, nkv;
  float eps;
};

constexpr int kRopeHeadsPerWarp = 8;  // heads of a token <= 8 warps x 8
// One CTA of 8 warps per prompt token (position s of sequence i), its warps taking the token's heads in
// turn (q heads, then k, then v); lane l holds elements 4l..4l+3, so the RoPE partner of element r
// (r ^ 64) sits in lane l ^ 16. The position's cos / sin entries are loaded once per lane. Same
// arithmetic and rounding points as the decode QKV epilogue (engine/kernels/fused.py:23-81 with
// pos_mode 0: position = prompt index).
__global__ void __launch_bounds__(256) prefill_qk_rope_kernel(const __grid_constant__ QkRopeArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t t = blockIdx.x;
  const int64_t i = t / a.S;
  int64_t s = t - i * a.S + a.pos0;  // s: the token's position (and cache slot)
  bool store_kv = true;
  if (a.slot0) {  // the sequence's slots start at slot0[i]: all S of them must lie in the cache
    const int64_t s0 = a.slot0[i];
    s = s0 + (t - i * a.S);
    if (s0 < 0 || s0 + a.S > a.cap) {
      if (threadIdx.x == 0 && a.err) atomicOr(a.err, QD_DEVERR_POS);
      store_kv = false;
      s = 0;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int heads = a.nq + 2 * a.nkv;
  int64_t rp = s;  // RoPE position: the slot, or the caller's per-token position (a token-tree node's depth)
  if (a.rope_pos) {
    rp = a.rope_pos[t];
    if (rp < 0 || rp >= a.cap) {
      if (threadIdx.x == 0 && a.err) atomicOr(a.err, QD_DEVERR_POS);
      rp = rp < 0 ? 0 : a.cap - 1;
    }
  }
  const uint2 cv = *reinterpret_cast<const uint2*>(a.cos + rp * 128 + 4 * lane);
  const uint2 sv = *reinterpret_cast<const uint2*>(a.sin + rp * 128 + 4 * lane);
  const float cs[4] = {bf_lo(cv.x), bf_hi(cv.x), bf_lo(cv.y), bf_hi(cv.y)};
  const float sn[4] = {bf_lo(sv.x), bf_hi(sv.x), bf_lo(sv.y), bf_hi(sv.y)};
  const uint2 qw = *reinterpret_cast<const uint2*>(a.qn + 4 * lane);
  const uint2 kw = *reinterpret_cast<const uint2*>(a.kn + 4 * lane);
  const __nv_bfloat16* row = a.qkv + t * a.ldqkv + 4 * lane;
  uint2 uu[kRopeHeadsPerWarp];  // every load of this warp's heads in flight before the first is used
#pragma unroll
  for (int j = 0; j < kRopeHeadsPerWarp; ++j) {
    const int h = warp + 8 * j;
    uu[j] = h < heads ? *reinterpret_cast<const uint2*>(row + (int64_t)h * 128) : make_uint2(0u, 0u);
  }
#pragma unroll
  for (int j = 0; j < kRopeHeadsPerWarp; ++j) {
    const int h = warp + 8 * j;
    if (h >= heads) break;
    const uint2 u = uu[j];
    if (h >= a.nq + a.nkv) {  // V head: into the cache as is
      const int kvh = h - a.nq - a.nkv;
      if (store_kv) *reinterpret_cast<uint2*>(a.v_cache + i * a.cs_b + kvh * a.cs_h + s * 128 + 4 * lane) = u;
      continue;
    }
    const float x[4] = {bf_lo(u.x), bf_hi(u.x), bf_lo(u.y), bf_hi(u.y)};
    const uint2 wv = h < a.nq ? qw : kw;
    const float nw[4] = {bf_lo(wv.x), bf_hi(wv.x), bf_lo(wv.y), bf_hi(wv.y)};
    float sq = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    sq = warp_sum(sq);
    const float rstd = 1.0f / sqrtf(sq / 128.0f + a.eps);
    float y[4], yp[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) y[e] = bf16r(nw[e] * bf16r(x[e] * rstd));
#pragma unroll
    for (int e = 0; e < 4; ++e) yp[e] = __shfl_xor_sync(0xffffffffu, y[e], 16);
    uint32_t o[2];
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      float r2[2];
#pragma unroll
      for (int d = 0; d < 2; ++d) {
        // q*cos + rotate_half(q)*sin with every product a BF16 tensor (rotate_half = cat(-q2, q1))
        const float rot = (lane < 16) ? bf16r(-yp[e + d] * sn[e + d]) : bf16r(yp[e + d] * sn[e + d]);
        r2[d] = bf16r(y[e + d] * cs[e + d]) + rot;
      }
      o[e >> 1] = pack_bf2(r2[0], r2[1]);
    }
    const uint2 ov = make_uint2(o[0], o[1]);
    if (h < a.nq)
      *reinterpret_cast<uint2*>(a.q_out + t * a.ldq + (int64_t)h * 128 + 4 * lane) = ov;
    else if (store_kv)
      *reinterpret_cast<uint2*>(a.k_cache + i * a.cs_b + (h - a.nq) * a.cs_h + s * 128 + 4 * lane) = ov;
  }
}

// ------------------------------------------------------------------ prompt causal attention
// Flash attention over the prompt (engine/engine.py:579, F.scaled_dot_product_attention with
// is_causal and enable_gqa) on the tensor cores, for the query positions q0..S-1 of every sequence
// (q0 = 0: the whole prompt; q0 = S - 1: the last layer, where only the last position continues,
// engine/engine.py:577-583). Work unit = (sequence, query head, tile of 128 queries); the units of the
// most key tiles go first. Per key tile of 128 keys:
//   S = Q K^T      tcgen05.mma M = 128 queries, N = 128 keys, K = 128 dims (8 MMAs), fp32 in TMEM,
//                  two S buffers so the next tile's S overlaps this tile's softmax
//   softmax        warps 0-7, two per query row (TMEM lane), each with 64 of the keys: row max
//                  (causal mask on the diagonal tile) from both halves' maxima exchanged through
//                  shared memory, then each turns its 64 keys into
//                  P = exp2((s - m) * scale * log2 e) (ex2.approx), rounded to BF16 into a
//                  128-byte-swizzled K-major operand tile (two P buffers), and sums them in fp32
//   O += P V       M = 128 queries, N = 128 dims (V read as an MN-major operand), K = 128 keys
// The running max only moves when some row of a warp grows by more than 2^8 in the exp2 domain; then
// the warp rescales its O columns in TMEM (tcgen05.ld / st) and its sums with them - the quotient
// O / l does not depend on which max is used. K and V have separate two-stage rings: a K tile is free
// once its S is computed, a V tile once its P.V is. Q, K and V arrive by TMA from tensor maps whose
// query / key extent is the prompt length, so rows past it read as zero. Warp 8 loads, warp 9 issues
// the MMAs.
constexpr int kPaThreads = 320;
constexpr int kPaTile = 128;
constexpr int kPaBox = kPaTile * 128;  // [128 rows][64 dims] BF16: 16 KiB

struct alignas(64) PrefillAttnArgs {
  CUtensorMap tq, tk, tv;
  __nv_bfloat16* out;  // [b * (S - q0), nq * 128]: row i * (S - q0) + s - q0
  int64_t ldo, S, q0;
  int batch, nq, nkv, n_qt, qt0, units;
  int qrow0;  // q tensor-map row of position 0 is -qrow0 (0: q holds every position; q0: only q0..S-1)
  float scale_log2;
  int* err;
  // token-tree rows (optional): the rows q0..S-1 are the nodes of one draft tree (S - q0 <= 32), and key
  // q0 + j is visible to the row at position q only if bit j of anc[q - q0] is set (its ancestors and
  // itself); keys before q0 follow the causal rule
  const uint32_t* anc;
};

struct PaLayout {
  static constexpr int q = 0;                      // Q: 2 dim halves
  static constexpr int k = q + 2 * kPaBox;         // K: 2 stages x 2 dim halves
  static constexpr int v = k + 2 * 2 * kPaBox;     // V: 2 stages x 2 dim halves
  static constexpr int p = v + 2 * 2 * kPaBox;     // P: 2 buffers x 2 key halves
  static constexpr int red = p + 2 * 2 * kPaBox;   // row max / sum exchange [2 tiles][2 halves][128] fp32
  static constexpr int bars = red + 2 * 2 * 128 * 4;  // 19 barriers
  static constexpr int misc = bars + 19 * 8;       // tmem slot, abort, K tiles, V tiles, Q tiles issued
  static constexpr int total = misc + 32;
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d_pf(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w,
                                               uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar), "l"(policy)
      : "memory");
}

// three-input max (sm_100) and the hardware base-2 exponential (flush-to-zero; exp2(-inf) = 0)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void pa_unit(const PrefillAttnArgs& a, int u, int* i, int* h, int* qt) {
  const int per = a.batch * a.nq;
  *qt = a.n_qt - 1 - u / per;  // >= qt0
  const int rem = u % per;
  *i = rem / a.nq;
  *h = rem - *i * a.nq;
}

__global__ void __launch_bounds__(kPaThreads, 1) prefill_attn_kernel(const __grid_constant__ PrefillAttnArgs a) {
  grid_dep_wait();  // holds no tensor memory while it waits; lets the next kernel in once it does
  // the layout needs all but a few hundred bytes of the 227 KiB, so there is no room to realign: dynamic
  // shared memory starts 1 KiB-aligned on sm_100 (nothing static precedes it); if not, flag and do nothing
  extern __shared__ __align__(1024) char smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.err, kErrSmem);
    return;
  }
  char* smem = smem_raw;
  const uint32_t sb = smem_u32(smem);
  const uint32_t bars = sb + PaLayout::bars;
  const uint32_t qfull = bars, qempty = bars + 8, ofree = bars + 144;
  auto kfull = [&](int s) { return bars + 16 + 8u * s; };
  auto kempty = [&](int s) { return bars + 32 + 8u * s; };
  auto vfull = [&](int s) { return bars + 48 + 8u * s; };
  auto vempty = [&](int s) { return bars + 64 + 8u * s; };
  auto sfull = [&](int s) { return bars + 80 + 8u * s; };
  auto sfree = [&](int s) { return bars + 96 + 8u * s; };
  auto pfull = [&](int s) { return bars + 112 + 8u * s; };
  auto odone = [&](int s) { return bars + 128 + 8u * s; };
  int* misc = reinterpret_cast<int*>(smem + PaLayout::misc);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  if (tid == 0) {
    mbar_init(qfull, 1);
    mbar_init(qempty, 1);
    mbar_init(ofree, 8);
    for (int s2 = 0; s2 < 2; ++s2) {
      mbar_init(kfull(s2), 1);
      mbar_init(kempty(s2), 1);
      mbar_init(vfull(s2), 1);
      mbar_init(vempty(s2), 1);
      mbar_init(sfull(s2), 1);
      mbar_init(sfree(s2), 8);
      mbar_init(pfull(s2), 8);
      mbar_init(odone(s2), 1);
    }
    fence_mbar_init();
    for (int m = 1; m < 8; ++m) misc[m] = 0;
  }
  if (warp == 9) tmem_alloc(smem_u32(misc), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_launch();
  const uint32_t tmem = (uint32_t)misc[0];
  const uint32_t tS = tmem, tO = tmem + 256;  // S[2] in columns 0-255, O in 256-383
  int* abort = misc + 1;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_normal();
      int t = 0, k = 0, kn = 0, vn = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < a.units && ok; u += G, ++k) {
        int i, h, qt;
        pa_unit(a, u, &i, &h, &qt);
        if (k >= 1 && !mbar_wait_abort(qempty, (k - 1) & 1, a.err, kErrWaitEmpty, abort)) break;
        misc[4] = k + 1;
        mbar_arrive_expect_tx(qfull, 2 * kPaBox);
        tma_load_3d(sb + PaLayout::q, &a.tq, h * 128, qt * kPaTile - a.qrow0, i, qfull, pol);
        tma_load_3d(sb + PaLayout::q + kPaBox, &a.tq, h * 128 + 64, qt * kPaTile - a.qrow0, i, qfull, pol);
        const int kvh = h / (a.nq / a.nkv);
        for (int j = 0; j <= qt; ++j, ++t) {
          const int st = t & 1;
          if (t >= 2 && !mbar_wait_abort(kempty(st), ((t >> 1) - 1) & 1, a.err, kErrWaitEmpty, abort)) {
            ok = false;
            break;
          }
          const uint32_t dk = sb + PaLayout::k + st * 2 * kPaBox;
          mbar_arrive_expect_tx(kfull(st), 2 * kPaBox);
          tma_load_4d_pf(dk, &a.tk, 0, j * kPaTile, kvh, i, kfull(st), pol);
          tma_load_4d_pf(dk + kPaBox, &a.tk, 64, j * kPaTile, kvh, i, kfull(st), pol);
          misc[2] = ++kn;
          if (t >= 2 && !mbar_wait_abort(vempty(st), ((t >> 1) - 1) & 1, a.err, kErrWaitEmpty, abort)) {
            ok = false;
            break;
          }
          const uint32_t dv = sb + PaLayout::v + st * 2 * kPaBox;
          mbar_arrive_expect_tx(vfull(st), 2 * kPaBox);
          tma_load_4d_pf(dv, &a.tv, 0, j * kPaTile, kvh, i, vfull(st), pol);
          tma_load_4d_pf(dv + kPaBox, &a.tv, 64, j * kPaTile, kvh, i, vfull(st), pol);
          misc[3] = ++vn;
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = umma_idesc_bf16(128), id_o = umma_idesc_bf16(128, false, true);
      int t = 0, k = 0;
      bool ok = true;
      auto issue_pv = [&](int tt, bool first) {
        const int b = tt & 1;
        if (ok && first && k >= 1) ok = mbar_wait_abort(ofree, (k - 1) & 1, a.err, kErrWaitFull, abort);
        if (ok) ok = mbar_wait_abort(pfull(b), (tt >> 1) & 1, a.err, kErrWaitFull, abort);
        if (ok) ok = mbar_wait_abort(vfull(b), (tt >> 1) & 1, a.err, kErrWaitFull, abort);
        tc_fence_after();
        if (ok) {
          const uint32_t v = sb + PaLayout::v + b * 2 * kPaBox, pp = sb + PaLayout::p + b * 2 * kPaBox;
#pragma unroll
          for (int j = 0; j < 8; ++j)  // 16 keys per MMA: P +32 B inside a 64-key half; V two 8-key atoms
            umma_bf16(tO, umma_desc_sw128(pp + (j >> 2) * kPaBox + (j & 3) * 32),
                      umma_desc_sw128(v + j * 2048, kPaBox, 1024), id_o, (first && j == 0) ? 0u : 1u);
        }
        umma_commit(odone(b));
        umma_commit(vempty(b));
      };
      for (int u = blockIdx.x; u < a.units && ok; u += G, ++k) {
        int i, h, qt;
        pa_unit(a, u, &i, &h, &qt);
        if (!mbar_wait_abort(qfull, k & 1, a.err, kErrWaitFull, abort)) break;
        for (int j = 0; j <= qt; ++j) {
          const int tt = t + j, b = tt & 1;
          if (ok) ok = mbar_wait_abort(kfull(b), (tt >> 1) & 1, a.err, kErrWaitFull, abort);
          if (ok && tt >= 2) ok = mbar_wait_abort(sfree(b), ((tt >> 1) - 1) & 1, a.err, kErrWaitFull, abort);
          tc_fence_after();
          if (ok) {
            const uint32_t kt = sb + PaLayout::k + b * 2 * kPaBox;
#pragma unroll
            for (int d = 0; d < 8; ++d)  // 16 dims per MMA: +32 B inside a 64-dim half, the next half after 4
              umma_bf16(tS + b * 128, umma_desc_sw128(sb + PaLayout::q + (d >> 2) * kPaBox + (d & 3) * 32),
                        umma_desc_sw128(kt + (d >> 2) * kPaBox + (d & 3) * 32), id_s, d > 0 ? 1u : 0u);
          }
          umma_commit(sfull(b));
          umma_commit(kempty(b));
          if (j == qt) umma_commit(qempty);
          if (j >= 1) issue_pv(tt - 1, j == 1);
        }
        issue_pv(t + qt, qt == 0);
        t += qt + 1;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue: two warps per row
    const int grp = warp >> 2, wq = warp & 3;  // grp: which 64 keys / dims of the row
    const int r = 32 * wq + lane;
    const uint32_t lane_off = (uint32_t)(32 * wq) << 16;
    float* red = reinterpret_cast<float*>(smem + PaLayout::red);
    int t = 0, k = 0;
    bool ok = true;
    // every softmax warp runs all its units and tiles even after a failed wait (the waits are then
    // skipped): the two warps of a row meet at named barriers, so neither may leave early
    for (int u = blockIdx.x; u < a.units; u += G, ++k) {
      int i, h, qt;
      pa_unit(a, u, &i, &h, &qt);
      const int q = qt * kPaTile + r;  // query position within the sequence
      // a token-tree row's ancestor mask over the keys q0.. (every key for rows outside the tree)
      const uint32_t tmask = (a.anc && q >= a.q0 && q < a.S) ? __ldg(a.anc + (q - a.q0)) : 0xffffffffu;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j <= qt; ++j) {
        const int tt = t + j, b = tt & 1;
        const uint32_t ts = tS + b * 128 + lane_off;
        if (ok) ok = mbar_wait_abort(sfull(b), (tt >> 1) & 1, a.err, kErrWaitFull, abort);
        tc_fence_after();
        const bool diag = (j == qt);
        // this half's 64 scores stay in registers for the exp pass; on the diagonal tile the keys past
        // the row's query (column > r) become -inf, whose exp2 is 0
        uint32_t own[64];
        tmem_ld64(ts + 64 * grp, own);
        if (diag) {
#pragma unroll
          for (int e = 0; e < 64; ++e)
            if (64 * grp + e > r) own[e] = __float_as_uint(-INFINITY);
        }
        if (a.anc && (int64_t)kPaTile * (j + 1) > a.q0) {  // tree keys in this tile: the ancestor mask
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const int64_t bit = (int64_t)kPaTile * j + 64 * grp + e - a.q0;
            if (bit >= 0 && bit < 32 && !((tmask >> bit) & 1u)) own[e] = __float_as_uint(-INFINITY);
          }
        }
        float mx;
        {  // four independent max chains
          float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int e = 0; e < 64; e += 8)
#pragma unroll
            for (int c = 0; c < 4; ++c)
              m4[c] = fmax3(m4[c], __uint_as_float(own[e + 2 * c]), __uint_as_float(own[e + 2 * c + 1]));
          mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        }
        {  // row max = max of the two halves' maxima (exchange slots alternate by tile)
          float* rx = red + b * 256;
          rx[grp * 128 + r] = mx;
          named_bar(1 + wq, 64);
          mx = fmaxf(rx[r], rx[128 + r]);
        }
        const float m_new = mx * a.scale_log2;
        // warp-uniform: the TMEM loads / stores of the rescale are warp-collective, and warps w and
        // w + 4 (the two halves of the same rows) take the same decision
        if (__any_sync(0xffffffffu, m_new > m_used + 8.f)) {
          const float m_to = fmaxf(m_used, m_new);
          const float alpha = exp2f(m_used - m_to);  // 0 on the first tile, 1 where the max did not grow
          if (j > 0) {
            // O must hold the previous tile's P.V before it is rescaled
            if (ok) ok = mbar_wait_abort(odone((tt - 1) & 1), ((tt - 1) >> 1) & 1, a.err, kErrWaitFull, abort);
            tc_fence_after();
#pragma unroll 1
            for (int c2 = 0; c2 < 2; ++c2) {
              const uint32_t ta = tO + lane_off + 64 * grp + 32 * c2;
              uint32_t o[32];
              tmem_ld32(ta, o);
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st32(ta, o);
            }
          }
          l *= alpha;
          m_used = m_to;
        }
        // P buffer b was last read by the P.V two tiles back
        if (ok && tt >= 2) ok = mbar_wait_abort(odone(b), ((tt >> 1) - 1) & 1, a.err, kErrWaitFull, abort);
        char* pt = smem + PaLayout::p + b * 2 * kPaBox + grp * kPaBox + r * 128;  // keys 64 grp.. of row r
        const float nm = -m_used;
        float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // eight independent sum chains
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 16-byte chunk c of the row (8 keys), stored swizzled by row
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const float p0 = ex2_approx(fmaf(__uint_as_float(own[8 * c + e]), a.scale_log2, nm));
            const float p1 = ex2_approx(fmaf(__uint_as_float(own[8 * c + e + 1]), a.scale_log2, nm));
            ls[e] += p0;
            ls[e + 1] += p1;
            pk[e >> 1] = pack_bf2(p0, p1);
          }
          *reinterpret_cast<uint4*>(pt + ((c ^ (r & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
        l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(sfree(b));
          mbar_arrive(pfull(b));
        }
      }
      // ---- unit end: O / l for this row's 64 dims; l is the sum of both halves
      const int tl = t + qt;
      if (ok) ok = mbar_wait_abort(odone(tl & 1), (tl >> 1) & 1, a.err, kErrWaitFull, abort);
      tc_fence_after();
      // the exchange slots of the tile after tl: both halves read them last before tile tl's barrier,
      // and the second barrier keeps the next tile's max from overwriting them before both have read
      float* lx = red + ((tl + 1) & 1) * 256;
      lx[grp * 128 + r] = l;
      named_bar(1 + wq, 64);
      const float inv = 1.0f / (lx[r] + lx[128 + r]);
      named_bar(1 + wq, 64);
      __nv_bfloat16* dst = a.out + ((int64_t)i * (a.S - a.q0) + (q - a.q0)) * a.ldo + (int64_t)h * 128 + 64 * grp;
#pragma unroll 1
      for (int c2 = 0; c2 < 2; ++c2) {
        uint32_t o[32];
        tmem_ld32(tO + lane_off + 64 * grp + 32 * c2, o);
        if (q < a.S && q >= a.q0) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c2);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            d4[c] = make_uint4(pack_bf2(__uint_as_float(o[8 * c]) * inv, __uint_as_float(o[8 * c + 1]) * inv),
                               pack_bf2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv),
                               pack_bf2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv),
                               pack_bf2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ofree);
      t += qt + 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, 512);
  if (tid == 0) {  // no bulk copy may still be writing shared memory when the CTA exits
    const int kn = misc[2], vn = misc[3], qn = misc[4];
    for (int it = kn > 2 ? kn - 2 : 0; it < kn; ++it)
      if (!mbar_wait(kfull(it & 1), (it >> 1) & 1, a.err, kErrDrain)) break;
    for (int it = vn > 2 ? vn - 2 : 0; it < vn; ++it)
      if (!mbar_wait(vfull(it & 1), (it >> 1) & 1, a.err, kErrDrain)) break;
    if (qn > 0) mbar_wait(qfull, (qn - 1) & 1, a.err, kErrDrain);
  }
}

// ------------------------------------------------------------------ prompt causal attention, ping-pong
// Variant of prefill_attn_kernel with two query tiles per CTA: query heads 2hp and 2hp + 1 of one KV
// head's group, same 128 queries, so both read every K / V tile the CTA loads. Two softmax warpgroups
// (warps 0-3 tile A, 4-7 tile B; thread = query row, all 128 keys of a tile in registers) alternate
// with the tensor core: while one warpgroup computes its P, the MMA warp runs the other tile's P.V and
// the next S. P is written back over its own S columns in tensor memory (BF16 pairs, 64 columns) and
// read from there as the A operand of P.V, so shared memory holds only Q (two tiles), and two K and
// two V stages. Tensor memory: S_A, S_B (128 columns each), O_A, O_B (128 each).
constexpr int kPpThreads = 320;

struct PpLayout {
  static constexpr int qa = 0;                  // Q of tile A: 2 dim halves
  static constexpr int qb = qa + 2 * kPaBox;    // Q of tile B
  static constexpr int k = qb + 2 * kPaBox;     // K: 2 stages x 2 dim halves
  static constexpr int v = k + 2 * 2 * kPaBox;  // V: 2 stages x 2 dim halves
  static constexpr int bars = v + 2 * 2 * kPaBox;
  static constexpr int nbars = 17;  // qfull, qempty, kfull[2], kempty[2], vfull[2], vempty[2], sfull[2],
                                    // pfull[2], odone[2], ofree
  static constexpr int misc = bars + nbars * 8;  // tmem slot, abort, K tiles, V tiles, Q units issued
  static constexpr int total = misc + 32;
};

__device__ __forceinline__ void pp_unit(const PrefillAttnArgs& a, int u, int* i, int* kvh, int* hp, int* qt) {
  const int per = a.batch * a.nkv * 2;
  *qt = a.n_qt - 1 - u / per;  // >= qt0
  const int rem = u % per;
  *i = rem / (a.nkv * 2);
  const int rr = rem - *i * a.nkv * 2;
  *kvh = rr >> 1;
  *hp = rr & 1;
}

__global__ void __launch_bounds__(kPpThreads, 1) prefill_attn_pp_kernel(const __grid_constant__ PrefillAttnArgs a) {
  grid_dep_wait();  // holds no tensor memory while it waits; lets the next kernel in once it does
  extern __shared__ __align__(1024) char smem_raw[];
  char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sb = smem_u32(smem);
  const uint32_t bars = sb + PpLayout::bars;
  const uint32_t qfull = bars, qempty = bars + 8, ofree = bars + 128;
  auto kfull = [&](int s) { return bars + 16 + 8u * s; };
  auto kempty = [&](int s) { return bars + 32 + 8u * s; };
  auto vfull = [&](int s) { return bars + 48 + 8u * s; };
  auto vempty = [&](int s) { return bars + 64 + 8u * s; };
  auto sfull = [&](int x) { return bars + 80 + 8u * x; };
  auto pfull = [&](int x) { return bars + 96 + 8u * x; };
  auto odone = [&](int x) { return bars + 112 + 8u * x; };
  static_assert(PpLayout::nbars * 8 == 136, "barrier block: 17 barriers");
  int* misc = reinterpret_cast<int*>(smem + PpLayout::misc);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, gq = a.nq / a.nkv;
  if (tid == 0) {
    mbar_init(qfull, 1);
    mbar_init(qempty, 1);
    mbar_init(ofree, 8);
    for (int s2 = 0; s2 < 2; ++s2) {
      mbar_init(kfull(s2), 1);
      mbar_init(kempty(s2), 1);
      mbar_init(vfull(s2), 1);
      mbar_init(vempty(s2), 1);
      mbar_init(sfull(s2), 1);
      mbar_init(pfull(s2), 4);
      mbar_init(odone(s2), 1);
    }
    fence_mbar_init();
    for (int m = 1; m < 8; ++m) misc[m] = 0;
  }
  if (warp == 9) tmem_alloc(smem_u32(misc), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_launch();
  const uint32_t tmem = (uint32_t)misc[0];
  auto tS = [&](int x) { return tmem + 128u * x; };        // S_A 0-127, S_B 128-255 (P over their first 64)
  auto tO = [&](int x) { return tmem + 256u + 128u * x; };  // O_A 256-383, O_B 384-511
  int* abort = misc + 1;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_normal();
      int t = 0, k = 0, kn = 0, vn = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < a.units && ok; u += G, ++k) {
        int i, kvh, hp, qt;
        pp_unit(a, u, &i, &kvh, &hp, &qt);
        if (k >= 1 && !mbar_wait_abort(qempty, (k - 1) & 1, a.err, kErrWaitEmpty, abort)) break;
        misc[4] = k + 1;
        const int ha = kvh * gq + 2 * hp;
        mbar_arrive_expect_tx(qfull, 4 * kPaBox);
        tma_load_3d(sb + PpLayout::qa, &a.tq, ha * 128, qt * kPaTile - a.qrow0, i, qfull, pol);
        tma_load_3d(sb + PpLayout::qa + kPaBox, &a.tq, ha * 128 + 64, qt * kPaTile - a.qrow0, i, qfull, pol);
        tma_load_3d(sb + PpLayout::qb, &a.tq, (ha + 1) * 128, qt * kPaTile - a.qrow0, i, qfull, pol);
        tma_load_3d(sb + PpLayout::qb + kPaBox, &a.tq, (ha + 1) * 128 + 64, qt * kPaTile - a.qrow0, i, qfull, pol);
        for (int j = 0; j <= qt; ++j, ++t) {
          const int st = t & 1;
          if (t >= 2 && !mbar_wait_abort(kempty(st), ((t >> 1) - 1) & 1, a.err, kErrWaitEmpty, abort)) {
            ok = false;
            break;
          }
          const uint32_t dk = sb + PpLayout::k + st * 2 * kPaBox;
          mbar_arrive_expect_tx(kfull(st), 2 * kPaBox);
          tma_load_4d_pf(dk, &a.tk, 0, j * kPaTile, kvh, i, kfull(st), pol);
          tma_load_4d_pf(dk + kPaBox, &a.tk, 64, j * kPaTile, kvh, i, kfull(st), pol);
          misc[2] = ++kn;
          if (t >= 2 && !mbar_wait_abort(vempty(st), ((t >> 1) - 1) & 1, a.err, kErrWaitEmpty, abort)) {
            ok = false;
            break;
          }
          const uint32_t dv = sb + PpLayout::v + st * 2 * kPaBox;
          mbar_arrive_expect_tx(vfull(st), 2 * kPaBox);
          tma_load_4d_pf(dv, &a.tv, 0, j * kPaTile, kvh, i, vfull(st), pol);
          tma_load_4d_pf(dv + kPaBox, &a.tv, 64, j * kPaTile, kvh, i, vfull(st), pol);
          misc[3] = ++vn;
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = umma_idesc_bf16(128), id_o = umma_idesc_bf16(128, false, true);
      int t = 0, k = 0;
      bool ok = true;
      auto issue_s = [&](int x, int tt) {  // S_x(tt) = Q_x K_tt^T; its columns then hold P_x(tt - 1) no more
        if (ok && tt > 0) ok = mbar_wait_abort(odone(x), (tt - 1) & 1, a.err, kErrWaitFull, abort);
        tc_fence_after();
        if (ok) {
          const uint32_t q = sb + (x ? PpLayout::qb : PpLayout::qa), kt = sb + PpLayout::k + (tt & 1) * 2 * kPaBox;
#pragma unroll
          for (int d = 0; d < 8; ++d)  // 16 dims per MMA: +32 B inside a 64-dim half, the next half after 4
            umma_bf16(tS(x), umma_desc_sw128(q + (d >> 2) * kPaBox + (d & 3) * 32),
                      umma_desc_sw128(kt + (d >> 2) * kPaBox + (d & 3) * 32), id_s, d > 0 ? 1u : 0u);
        }
        umma_commit(sfull(x));
      };
      auto issue_pv = [&](int x, int tt, bool first) {  // O_x += P_x(tt) V_tt, P from tensor memory
        if (ok) ok = mbar_wait_abort(pfull(x), tt & 1, a.err, kErrWaitFull, abort);
        tc_fence_after();
        if (ok) {
          const uint32_t v = sb + PpLayout::v + (tt & 1) * 2 * kPaBox;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // 16 keys per MMA: 8 columns of P pairs; V two 8-key atoms
            umma_bf16_ts(tO(x), tS(x) + 8 * kk, umma_desc_sw128(v + kk * 2048, kPaBox, 1024), id_o,
                         (first && kk == 0) ? 0u : 1u);
        }
        umma_commit(odone(x));
      };
      for (int u = blockIdx.x; u < a.units && ok; u += G, ++k) {
        int i, kvh, hp, qt;
        pp_unit(a, u, &i, &kvh, &hp, &qt);
        const int J = qt + 1;
        if (!mbar_wait_abort(qfull, k & 1, a.err, kErrWaitFull, abort)) break;
        if (ok) ok = mbar_wait_abort(kfull(t & 1), (t >> 1) & 1, a.err, kErrWaitFull, abort);
        issue_s(0, t);
        issue_s(1, t);
        umma_commit(kempty(t & 1));
        if (J == 1) umma_commit(qempty);
        for (int j = 0; j < J; ++j) {
          const int tt = t + j;
          if (ok && j == 0 && k >= 1) ok = mbar_wait_abort(ofree, (k - 1) & 1, a.err, kErrWaitFull, abort);
          if (ok) ok = mbar_wait_abort(vfull(tt & 1), (tt >> 1) & 1, a.err, kErrWaitFull, abort);
          issue_pv(0, tt, j == 0);
          if (j + 1 < J) {
            if (ok) ok = mbar_wait_abort(kfull((tt + 1) & 1), ((tt + 1) >> 1) & 1, a.err, kErrWaitFull, abort);
            issue_s(0, tt + 1);
          }
          issue_pv(1, tt, j == 0);
          umma_commit(vempty(tt & 1));
          if (j + 1 < J) {
            issue_s(1, tt + 1);
            umma_commit(kempty((tt + 1) & 1));
            if (j + 2 == J) umma_commit(qempty);
          }
        }
        t += J;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue: warpgroup x = tile x
    const int x = warp >> 2, wq = warp & 3, r = 32 * wq + lane;
    const uint32_t lane_off = (uint32_t)(32 * wq) << 16;
    int t = 0, k = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < a.units; u += G, ++k) {
      int i, kvh, hp, qt;
      pp_unit(a, u, &i, &kvh, &hp, &qt);
      const int h = kvh * gq + 2 * hp + x;
      const int q = qt * kPaTile + r;  // query position within the sequence
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j <= qt; ++j) {
        const int tt = t + j;
        if (ok) ok = mbar_wait_abort(sfull(x), tt & 1, a.err, kErrWaitFull, abort);
        tc_fence_after();
        uint32_t sv[128];
        tmem_ld64(tS(x) + lane_off, sv);
        tmem_ld64(tS(x) + lane_off + 64, sv + 64);
        if (j == qt) {  // diagonal tile: keys past the row's query (column > r) do not count
#pragma unroll
          for (int e = 0; e < 128; ++e)
            if (e > r) sv[e] = __float_as_uint(-INFINITY);
        }
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int e = 0; e < 128; e += 8)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            m4[c] = fmax3(m4[c], __uint_as_float(sv[e + 2 * c]), __uint_as_float(sv[e + 2 * c + 1]));
        const float m_new = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * a.scale_log2;
        // warp-uniform (the TMEM loads / stores of the rescale are warp-collective); O_x holds P.V up to
        // tile tt - 1 (S_x(tt) was issued after it completed) and P.V of tile tt has not started
        if (__any_sync(0xffffffffu, m_new > m_used + 8.f)) {
          const float m_to = fmaxf(m_used, m_new);
          const float alpha = exp2f(m_used - m_to);  // 0 on the first tile, 1 where the max did not grow
          if (j > 0) {
#pragma unroll 1
            for (int c4 = 0; c4 < 4; ++c4) {
              uint32_t o[32];
              tmem_ld32(tO(x) + lane_off + 32 * c4, o);
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st32(tO(x) + lane_off + 32 * c4, o);
            }
          }
          l *= alpha;
          m_used = m_to;
        }
        const float nm = -m_used;
        float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 64; ++c) {  // P pair c = keys 2c, 2c + 1, packed in place over the scores
          const float p0 = ex2_approx(fmaf(__uint_as_float(sv[2 * c]), a.scale_log2, nm));
          const float p1 = ex2_approx(fmaf(__uint_as_float(sv[2 * c + 1]), a.scale_log2, nm));
          ls[(2 * c) & 7] += p0;
          ls[(2 * c + 1) & 7] += p1;
          sv[c] = pack_bf2(p0, p1);
        }
        l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
        tmem_st64(tS(x) + lane_off, sv);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pfull(x));
      }
      // ---- unit end: O / l for this row
      const int tl = t + qt;
      if (ok) ok = mbar_wait_abort(odone(x), tl & 1, a.err, kErrWaitFull, abort);
      tc_fence_after();
      const float inv = 1.0f / l;
      __nv_bfloat16* dst = a.out + ((int64_t)i * (a.S - a.q0) + (q - a.q0)) * a.ldo + (int64_t)h * 128;
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t o[32];
        tmem_ld32(tO(x) + lane_off + 32 * c4, o);
        if (q < a.S && q >= a.q0) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c4);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            d4[c] = make_uint4(pack_bf2(__uint_as_float(o[8 * c]) * inv, __uint_as_float(o[8 * c + 1]) * inv),
                               pack_bf2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv),
                               pack_bf2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv),
                               pack_bf2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ofree);
      t += qt + 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, 512);
  if (tid == 0) {  // no bulk copy may still be writing shared memory when the CTA exits
    const int kn = misc[2], vn = misc[3], qn = misc[4];
    for (int it = kn > 2 ? kn - 2 : 0; it < kn; ++it)
      if (!mbar_wait(kfull(it & 1), (it >> 1) & 1, a.err, kErrDrain)) break;
    for (int it = vn > 2 ? vn - 2 : 0; it < vn; ++it)
      if (!mbar_wait(vfull(it & 1), (it >> 1) & 1, a.err, kErrDrain)) break;
    if (qn > 0) mbar_wait(qfull, (qn - 1) & 1, a.err, kErrDrain);
  }
}

// ------------------------------------------------------------------ host side
template <int BN>
static int gemm_nst() {
  int nst = env_int("QD_GEMM_STAGES", 8);
  if (nst > 8) nst = 8;
  while (nst > 2 && GemmLayout<BN>::total(nst) + 1024 > 227 * 1024) --nst;
  return nst;
}

// BN = 256 when the 256-wide tiles alone give every SM at least one tile, else 128
static int gemm_bn(int64_t m, int64_t n) {
  const int64_t mt = (m + 127) / 128;
  const int forced = env_int("QD_GEMM_BN", 0);
  if (forced == 128 || forced == 256) return forced;
  return mt * ((n + 255) / 256) >= host_sm_count() ? 256 : 128;
}

// ---------------------------------------------------------------- split-K sum + epilogue
// For every split tile: out = epilogue(sum over splits s = 0, 1, .. of the fp32 partials, in that order),
// the same bits on every run. Block (x, y) = 256 threads over output quads (four consecutive columns) of
// split tile y, quad-fastest within a row; every split's float4 is in flight at once, so the partials
// (just written, still in L2) stream at full width. Launched right behind the GEMM (programmatic
// dependent launch); griddepcontrol.wait holds it until the GEMM's partials are visible.
constexpr int kMaxKsplit = 16;

struct SplitSumArgs {
  const float* partials;  // [split tiles][ksplit][128][bn]
  __nv_bfloat16* out;
  const __nv_bfloat16* res;
  int64_t ldo, ldr, m, n;
  int full_tiles, m_tiles, n_tiles, ngroups, ksplit;
  int bn_shift, qpt_shift;  // log2 tile width; log2 output quads per tile row
};

__device__ __forceinline__ float4 split_sum(const SplitSumArgs& a, const float* p) {
  const int64_t sstride = (int64_t)128 << a.bn_shift;
  float4 v[kMaxKsplit];
#pragma unroll
  for (int s = 0; s < kMaxKsplit; ++s)
    if (s < a.ksplit) v[s] = __ldcg(reinterpret_cast<const float4*>(p + s * sstride));
  float4 acc = v[0];
#pragma unroll
  for (int s = 1; s < kMaxKsplit; ++s)
    if (s < a.ksplit) {
      acc.x += v[s].x;
      acc.y += v[s].y;
      acc.z += v[s].z;
      acc.w += v[s].w;
    }
  return acc;
}

template <int EPI>
__global__ void __launch_bounds__(256) gemm_splitk_sum_kernel(const __grid_constant__ SplitSumArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int j = blockIdx.y;
  const int idx = blockIdx.x * 256 + threadIdx.x;
  const int r = idx >> a.qpt_shift, oc = (idx - (r << a.qpt_shift)) * 4;  // tile row; first output column
  if (r >= 128) return;
  int mt, nt;
  gemm_tile(a.m_tiles, a.n_tiles, a.full_tiles + j, &mt, &nt);
  const int64_t row = (int64_t)mt * 128 + r;
  if (row >= a.m) return;
  const int bn = 1 << a.bn_shift;
  const float* pt = a.partials + (((int64_t)j * a.ksplit) * 128 + r) * bn;
  float y[4];
  int64_t col;
  if constexpr (EPI == GEMM_SWIGLU) {
    // tile output column oc: group h = oc / 64 of the tile, gate at tile column 128 h + oc % 64, up 64 further
    const int h = oc >> 6, jj = oc & 63, g = nt * (bn >> 7) + h;
    if (g >= a.ngroups) return;  // the repeated last group of an odd group count
    const float4 g4 = split_sum(a, pt + h * 128 + jj), u4 = split_sum(a, pt + h * 128 + 64 + jj);
    const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, uv[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float gb = bf16r(gv[e]);
      y[e] = bf16r(gb / (1.0f + expf(-gb))) * bf16r(uv[e]);
    }
    col = (int64_t)g * 64 + jj;
  } else {
    col = (int64_t)nt * bn + oc;
    if (col >= a.n) return;
    const float4 s4 = split_sum(a, pt + oc);
    y[0] = bf16r(s4.x);
    y[1] = bf16r(s4.y);
    y[2] = bf16r(s4.z);
    y[3] = bf16r(s4.w);
    if constexpr (EPI == GEMM_RES) {
      const uint2 u = *reinterpret_cast<const uint2*>(a.res + row * a.ldr + col);
      y[0] += bf_lo(u.x);
      y[1] += bf_hi(u.x);
      y[2] += bf_lo(u.y);
      y[3] += bf_hi(u.y);
    }
  }
  *reinterpret_cast<uint2*>(a.out + row * a.ldo + col) = make_uint2(pack_bf2(y[0], y[1]), pack_bf2(y[2], y[3]));
}

// Stream-K style plan: the tiles that fill whole waves (tiles / SMs of them, x SMs) run whole; the tiles of
// the last, partial wave are split along K into as many ranges as keep them in one wave (at most SMs /
// remaining tiles, each >= 8 K-blocks, at most kMaxKsplit), so a short prompt's few tiles, or a ragged
// last wave, still spread over every SM. QD_GEMM_KSPLIT forces the split of every tile (1 = none).
// The scratch holds the split tiles' fp32 partials.
constexpr int64_t kGemmMaxSplitTiles = 1024;
struct GemmPlan {
  int bn, grid, ksplit;
  int64_t tiles, full_tiles, scratch_bytes;
};
static GemmPlan gemm_plan(int64_t m, int64_t n, int64_t k) {
  GemmPlan p;
  p.bn = gemm_bn(m, n);
  p.tiles = ((m + 127) / 128) * ((n + p.bn - 1) / p.bn);
  const int sms = host_sm_count();
  const int64_t kblocks = k / 64;
  const int64_t rem = p.tiles % sms;
  int64_t ks = rem ? sms / rem : 1;
  if (ks > kblocks / 8) ks = kblocks / 8;
  p.full_tiles = p.tiles - rem;
  const int forced = env_int("QD_GEMM_KSPLIT", 0);
  if (forced >= 1) {
    ks = forced > kblocks ? kblocks : forced;
    p.full_tiles = 0;
  }
  if (ks > kMaxKsplit) ks = kMaxKsplit;
  if (ks < 2 || p.tiles - p.full_tiles > kGemmMaxSplitTiles) {
    ks = 1;
    p.full_tiles = p.tiles;
  }
  p.ksplit = (int)ks;
  const int64_t units = p.full_tiles + (p.tiles - p.full_tiles) * ks;
  p.grid = (int)(units < sms ? units : sms);
  p.scratch_bytes = ks > 1 ? (p.tiles - p.full_tiles) * ks * 128 * p.bn * 4 : 0;
  return p;
}

template <int BN, int EPI>
static int launch_gemm(const GemmArgs& a, int grid, cudaStream_t stream) {
  auto kern = tc_gemm_kernel<BN, EPI>;
  const int smem = GemmLayout<BN>::total(a.nst) + 1024;
  if (int rc = set_max_dynamic_smem((const void*)kern, smem)) return rc;
  return launch_kernel((const void*)kern, dim3(grid), dim3(kGemmThreads), smem, 1, stream, (void*)&a);
}

}  // namespace qd

using namespace qd;

extern "C" int qd_tc_gemm_plan(int64_t m, int64_t n, int64_t k, int* grid, int* bn, int* ksplit,
                               int64_t* scratch_bytes) {
  if (m < 1 || n < 128 || n % 128 || k < 64 || k % 64) return set_error(QD_ERR_ARG, "tc gemm plan: bad sizes");
  const GemmPlan p = gemm_plan(m, n, k);
  if (grid) *grid = p.grid;
  if (bn) *bn = p.bn;
  if (ksplit) *ksplit = p.ksplit;
  if (scratch_bytes) *scratch_bytes = p.scratch_bytes;
  return QD_OK;
}

extern "C" int qd_tc_gemm(const void* x, int64_t ldx, int64_t m, const void* w_packed, int64_t n, int64_t k, void* out,
                          int64_t ldo, const void* res, int64_t ldr, int epilogue, void* scratch, int64_t scratch_bytes,
                          int* err, cudaStream_t stream) {
  if (!x || !w_packed || !out) return set_error(QD_ERR_ARG, "null pointer");
  if (m < 1 || n < 128 || n % 128 || k < 64 || k % 64 || ldx < k || ldx % 8 || ldo % 8)
    return set_error(QD_ERR_ARG, "tc gemm: m >= 1, n %% 128 == 0, k %% 64 == 0, ldx >= k, ldx/ldo %% 8 == 0");
  if (epilogue != GEMM_STORE && epilogue != GEMM_RES && epilogue != GEMM_SWIGLU)
    return set_error(QD_ERR_ARG, "tc gemm: epilogue must be QD_EPI_STORE, QD_EPI_RES or QD_EPI_SWIGLU");
  if (ldo < (epilogue == GEMM_SWIGLU ? n / 2 : n)) return set_error(QD_ERR_ARG, "tc gemm: ldo too small");
  if (epilogue == GEMM_RES && (!res || ldr < n || ldr % 8 || !aligned16(res)))
    return set_error(QD_ERR_ARG, "tc gemm: residual needs ldr >= n, ldr %% 8 == 0, 16-byte alignment");
  if (!aligned16(x) || !aligned16(w_packed) || !aligned16(out)) return set_error(QD_ERR_ARG, "tc gemm: alignment");
  if (m > (int64_t)INT32_MAX - 128 || k > (1 << 24)) return set_error(QD_ERR_UNSUPPORTED, "tc gemm: too large");
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return set_error(QD_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  GemmArgs a = {};
  {
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
    const cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(&a.tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(QD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  }
  const GemmPlan gp = gemm_plan(m, n, k);
  const int bn = gp.bn;
  if (gp.scratch_bytes > 0 && (!scratch || scratch_bytes < gp.scratch_bytes || !aligned16(scratch)))
    return set_error(QD_ERR_SCRATCH, "tc gemm: split-K needs %lld B of 16-byte aligned scratch (have %lld)",
                     (long long)gp.scratch_bytes, (long long)scratch_bytes);
  a.ksplit = gp.ksplit;
  a.partials = gp.ksplit > 1 ? static_cast<float*>(scratch) : nullptr;
  a.w = static_cast<const char*>(w_packed);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.res = static_cast<const __nv_bfloat16*>(res);
  a.ldo = ldo;
  a.ldr = ldr;
  a.m = m;
  a.n = n;
  a.kblocks = (int)(k / 64);
  a.ngroups = (int)(n / 128);
  a.m_tiles = (int)((m + 127) / 128);
  a.n_tiles = (int)((n + bn - 1) / bn);
  const int64_t tiles = (int64_t)a.m_tiles * a.n_tiles;
  if (tiles > INT32_MAX) return set_error(QD_ERR_UNSUPPORTED, "tc gemm: too many tiles");
  a.tiles = (int)tiles;
  const int64_t units = gp.full_tiles + (tiles - gp.full_tiles) * gp.ksplit;
  if (units > INT32_MAX) return set_error(QD_ERR_UNSUPPORTED, "tc gemm: too many work units");
  a.full_tiles = (int)gp.full_tiles;
  a.units = (int)units;
  a.err = err;
  const int grid = gp.grid;
  int rc;
  if (bn == 256) {
    a.nst = gemm_nst<256>();
    rc = epilogue == GEMM_STORE ? launch_gemm<256, GEMM_STORE>(a, grid, stream)
         : epilogue == GEMM_RES ? launch_gemm<256, GEMM_RES>(a, grid, stream)
                                : launch_gemm<256, GEMM_SWIGLU>(a, grid, stream);
  } else {
    a.nst = gemm_nst<128>();
    rc = epilogue == GEMM_STORE ? launch_gemm<128, GEMM_STORE>(a, grid, stream)
         : epilogue == GEMM_RES ? launch_gemm<128, GEMM_RES>(a, grid, stream)
                                : launch_gemm<128, GEMM_SWIGLU>(a, grid, stream);
  }
  if (rc != QD_OK || gp.ksplit == 1) return rc;
  SplitSumArgs sa = {};
  sa.partials = a.partials;
  sa.out = a.out;
  sa.res = a.res;
  sa.ldo = ldo;
  sa.ldr = ldr;
  sa.m = m;
  sa.n = n;
  sa.full_tiles = a.full_tiles;
  sa.m_tiles = a.m_tiles;
  sa.n_tiles = a.n_tiles;
  sa.ngroups = a.ngroups;
  sa.ksplit = gp.ksplit;
  sa.bn_shift = bn == 256 ? 8 : 7;
  sa.qpt_shift = sa.bn_shift - (epilogue == GEMM_SWIGLU ? 3 : 2);  // BN / 8 or BN / 4 quads per tile row
  const dim3 block(256), sgrid((unsigned)((128 << sa.qpt_shift) / 256), (unsigned)(tiles - gp.full_tiles));
  const void* kern = epilogue == GEMM_STORE ? (const void*)gemm_splitk_sum_kernel<GEMM_STORE>
                     : epilogue == GEMM_RES ? (const void*)gemm_splitk_sum_kernel<GEMM_RES>
                                            : (const void*)gemm_splitk_sum_kernel<GEMM_SWIGLU>;
  return launch_kernel(kern, sgrid, block, 0, 1, stream, &sa);
}

extern "C" int qd_rmsnorm_rows(const void* x, int64_t ldx, int64_t m, int64_t k, const void* norm_w, float eps,
                               void* out, int64_t ldo, cudaStream_t stream) {
  if (!x || !norm_w || !out) return set_error(QD_ERR_ARG, "null pointer");
  if (m < 1 || k < 8 || k % 8 || ldx < k || ldo < k || ldx % 8 || ldo % 8 || m > INT32_MAX)
    return set_error(QD_ERR_ARG, "rmsnorm: bad sizes");
  if (!aligned16(x) || !aligned16(norm_w) || !aligned16(out)) return set_error(QD_ERR_ARG, "rmsnorm: alignment");
  RmsArgs a = {};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.w = static_cast<const __nv_bfloat16*>(norm_w);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldx = ldx;
  a.ldo = ldo;
  a.k = k;
  a.eps = eps;
  return launch_kernel((const void*)rmsnorm_rows_kernel, dim3((unsigned)m), dim3(256), 0, 1, stream, &a);
}

extern "C" int qd_argmax_rows(const void* logits, int64_t ld, int64_t n, int64_t rows, int64_t* out,
                              cudaStream_t stream) {
  if (!logits || !out) return set_error(QD_ERR_ARG, "null pointer");
  if (rows < 1 || rows > INT32_MAX || n < 1 || ld < n || ld % 8) return set_error(QD_ERR_ARG, "argmax: bad sizes");
  if (!aligned16(logits)) return set_error(QD_ERR_ARG, "argmax: logits not 16-byte aligned");
  ArgmaxArgs a = {};
  a.logits = static_cast<const __nv_bfloat16*>(logits);
  a.out = out;
  a.ld = ld;
  a.n = n;
  return launch_kernel((const void*)argmax_rows_kernel, dim3((unsigned)rows), dim3(256), 0, 1, stream, &a);
}

extern "C" int qd_prefill_qk_rope(const void* qkv, int64_t ldqkv, int batch, int64_t S, int nq_heads, int nkv_heads,
                                  const void* q_norm, const void* k_norm, float eps, const void* cos, const void* sin,
                                  void* q_out, int64_t ldq, void* k_cache, void* v_cache, int64_t cap, int64_t cs_b,
                                  int64_t cs_h, cudaStream_t stream) {
  return qd_prefill_qk_rope_at(qkv, ldqkv, batch, S, 0, nq_heads, nkv_heads, q_norm, k_norm, eps, cos, sin, q_out, ldq,
                               k_cache, v_cache, cap, cs_b, cs_h, stream);
}

static int qk_rope(const void* qkv, int64_t ldqkv, int batch, int64_t S, int64_t pos0, const int32_t* slot0,
                   const int32_t* rope_pos, int nq_heads, int nkv_heads, const void* q_norm, const void* k_norm, float eps, const void* cos,
                   const void* sin, void* q_out, int64_t ldq, void* k_cache, void* v_cache, int64_t cap, int64_t cs_b,
                   int64_t cs_h, int* err, cudaStream_t stream) {
  if (!qkv || !q_norm || !k_norm || !cos || !sin || !q_out || !k_cache || !v_cache)
    return set_error(QD_ERR_ARG, "null pointer");
  if (pos0 < 0 || pos0 > cap) return set_error(QD_ERR_ARG, "prefill q/k rope: pos0 outside [0, cap]");
  if (batch < 1 || S < 1 || S > cap - pos0 || nq_heads < 1 || nkv_heads < 1 ||
      nq_heads + 2 * nkv_heads > 8 * kRopeHeadsPerWarp ||
      ldqkv < (int64_t)(nq_heads + 2 * nkv_heads) * 128 || ldq < (int64_t)nq_heads * 128 || ldqkv % 4 || ldq % 4 ||
      cs_h < cap * 128 || cs_b < (int64_t)nkv_heads * cs_h || cs_h % 4 || cs_b % 4)
    return set_error(QD_ERR_ARG, "prefill q/k rope: bad sizes");
  if (((uintptr_t)qkv | (uintptr_t)q_out | (uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)q_norm |
       (uintptr_t)k_norm | (uintptr_t)cos | (uintptr_t)sin) & 7)
    return set_error(QD_ERR_ARG, "prefill q/k rope: 8-byte alignment");
  QkRopeArgs a = {};
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.qn = static_cast<const __nv_bfloat16*>(q_norm);
  a.kn = static_cast<const __nv_bfloat16*>(k_norm);
  a.cos = static_cast<const __nv_bfloat16*>(cos);
  a.sin = static_cast<const __nv_bfloat16*>(sin);
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.ldqkv = ldqkv;
  a.ldq = ldq;
  a.S = S;
  a.cs_b = cs_b;
  a.cs_h = cs_h;
  a.tokens = (int64_t)batch * S;
  a.pos0 = pos0;
  a.nq = nq_heads;
  a.nkv = nkv_heads;
  a.eps = eps;
  a.rope_pos = rope_pos;
  a.slot0 = slot0;
  a.cap = cap;
  a.err = err;
  if (a.tokens > INT32_MAX) return set_error(QD_ERR_UNSUPPORTED, "prefill q/k rope: too many tokens");
  return launch_kernel((const void*)prefill_qk_rope_kernel, dim3((unsigned)a.tokens), dim3(256), 0, 1, stream, &a);
}

extern "C" int qd_prefill_qk_rope_at(const void* qkv, int64_t ldqkv, int batch, int64_t S, int64_t pos0, int nq_heads,
                                     int nkv_heads, const void* q_norm, const void* k_norm, float eps, const void* cos,
                                     const void* sin, void* q_out, int64_t ldq, void* k_cache, void* v_cache,
                                     int64_t cap, int64_t cs_b, int64_t cs_h, cudaStream_t stream) {
  return qk_rope(qkv, ldqkv, batch, S, pos0, nullptr, nullptr, nq_heads, nkv_heads, q_norm, k_norm, eps, cos, sin,
                 q_out, ldq, k_cache, v_cache, cap, cs_b, cs_h, nullptr, stream);
}

extern "C" int qd_tree_qk_rope(const void* qkv, int64_t ldqkv, int batch, int T, const int32_t* slot0,
                               const int32_t* rope_pos, int nq_heads, int nkv_heads, const void* q_norm,
                               const void* k_norm, float eps, const void* cos, const void* sin, void* q_out,
                               int64_t ldq, void* k_cache, void* v_cache, int64_t cap, int64_t cs_b, int64_t cs_h,
                               int* err, cudaStream_t stream) {
  if (!slot0 || !rope_pos) return set_error(QD_ERR_ARG, "tree q/k rope: null slot or position array");
  return qk_rope(qkv, ldqkv, batch, T, 0, slot0, rope_pos, nq_heads, nkv_heads, q_norm, k_norm, eps, cos, sin, q_out,
                 ldq, k_cache, v_cache, cap, cs_b, cs_h, err, stream);
}

static int prefill_attn(const void* q, int64_t ldq, int batch, int64_t S, int64_t q_begin, bool q_compact, int nq_heads,
                        int nkv_heads, const void* k_cache, const void* v_cache, int64_t cap, int64_t cs_b,
                        int64_t cs_h, float scale, void* out, int64_t ldo, int* err, cudaStream_t stream,
                        const uint32_t* anc = nullptr);

extern "C" int qd_prefill_attn(const void* q, int64_t ldq, int batch, int64_t S, int64_t q_begin, int nq_heads,
                               int nkv_heads, const void* k_cache, const void* v_cache, int64_t cap, int64_t cs_b,
                               int64_t cs_h, float scale, void* out, int64_t ldo, int* err, cudaStream_t stream) {
  return prefill_attn(q, ldq, batch, S, q_begin, false, nq_heads, nkv_heads, k_cache, v_cache, cap, cs_b, cs_h, scale,
                      out, ldo, err, stream);
}

extern "C" int qd_prefill_attn_rows(const void* q, int64_t ldq, int batch, int64_t S, int64_t q_begin, int nq_heads,
                                    int nkv_heads, const void* k_cache, const void* v_cache, int64_t cap, int64_t cs_b,
                                    int64_t cs_h, float scale, void* out, int64_t ldo, int* err, cudaStream_t stream) {
  return prefill_attn(q, ldq, batch, S, q_begin, true, nq_heads, nkv_heads, k_cache, v_cache, cap, cs_b, cs_h, scale,
                      out, ldo, err, stream);
}

extern "C" int qd_tree_attn_rows(const void* q, int64_t ldq, int64_t S, int64_t q_begin, const uint32_t* anc,
                                 int nq_heads, int nkv_heads, const void* k_cache, const void* v_cache, int64_t cap,
                                 int64_t cs_h, float scale, void* out, int64_t ldo, int* err, cudaStream_t stream) {
  if (!anc) return set_error(QD_ERR_ARG, "tree attention rows: null ancestor masks");
  if (S - q_begin < 1 || S - q_begin > 32) return set_error(QD_ERR_ARG, "tree attention rows: 1 to 32 tree rows");
  return prefill_attn(q, ldq, 1, S, q_begin, true, nq_heads, nkv_heads, k_cache, v_cache, cap,
                      (int64_t)nkv_heads * cs_h, cs_h, scale, out, ldo, err, stream, anc);
}

static int prefill_attn(const void* q, int64_t ldq, int batch, int64_t S, int64_t q_begin, bool q_compact, int nq_heads,
                        int nkv_heads, const void* k_cache, const void* v_cache, int64_t cap, int64_t cs_b,
                        int64_t cs_h, float scale, void* out, int64_t ldo, int* err, cudaStream_t stream,
                        const uint32_t* anc) {
  if (!q || !k_cache || !v_cache || !out) return set_error(QD_ERR_ARG, "null pointer");
  if (batch < 1 || S < 1 || S > cap || q_begin < 0 || q_begin >= S || nq_heads < 1 || nkv_heads < 1 ||
      nq_heads % nkv_heads || ldq < (int64_t)nq_heads * 128 || ldo < (int64_t)nq_heads * 128 || ldq % 8 ||
      ldo % 8 || cs_h < cap * 128 || cs_b < (int64_t)nkv_heads * cs_h || cs_h % 8 || cs_b % 8)
    return set_error(QD_ERR_ARG, "prefill attention: bad sizes or strides");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return set_error(QD_ERR_ARG, "prefill attention: alignment");
  const int64_t n_qt = (S + kPaTile - 1) / kPaTile, qt0 = q_begin / kPaTile;
  const int64_t units = (int64_t)batch * nq_heads * (n_qt - qt0);
  if (units > INT32_MAX || S > INT32_MAX - kPaTile) return set_error(QD_ERR_UNSUPPORTED, "prefill attention: too large");
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return set_error(QD_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  PrefillAttnArgs a = {};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  {
    // q rows of every sequence: positions 0..S-1, or (q_compact) only q_begin..S-1, loaded at row
    // coordinate position - qrow0 (the rows before q_begin of the first query tile read as zero)
    const int64_t qrows = q_compact ? S - q_begin : S;
    const cuuint64_t dims[3] = {(cuuint64_t)nq_heads * 128, (cuuint64_t)qrows, (cuuint64_t)batch};
    const cuuint64_t strides[2] = {(cuuint64_t)ldq * 2, (cuuint64_t)(qrows * ldq * 2)};
    const cuuint32_t box[3] = {64, (cuuint32_t)kPaTile, 1};
    if (encode(&a.tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return set_error(QD_ERR_CUDA, "cuTensorMapEncodeTiled failed for q");
  }
  {
    // key extent = the prompt length: keys past it read as zero
    const cuuint64_t dims[4] = {128, (cuuint64_t)S, (cuuint64_t)nkv_heads, (cuuint64_t)batch};
    const cuuint64_t strides[3] = {256, (cuuint64_t)cs_h * 2, (cuuint64_t)cs_b * 2};
    const cuuint32_t box[4] = {64, (cuuint32_t)kPaTile, 1, 1};
    if (encode(&a.tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(k_cache), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        encode(&a.tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(v_cache), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return set_error(QD_ERR_CUDA, "cuTensorMapEncodeTiled failed for the KV cache");
  }
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.S = S;
  a.q0 = q_begin;
  a.qrow0 = q_compact ? (int)q_begin : 0;
  a.qt0 = (int)qt0;
  a.batch = batch;
  a.nq = nq_heads;
  a.nkv = nkv_heads;
  a.n_qt = (int)n_qt;
  a.units = (int)units;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = err;
  a.anc = anc;
  if (!anc && env_int("QD_PREFILL_ATTN", 1) == 2 && (nq_heads / nkv_heads) % 2 == 0) {  // ping-pong variant
    a.units = (int)(units / 2);  // a unit covers two query heads of one KV head
    const int smem = PpLayout::total + 1024;
    if (int rc = set_max_dynamic_smem((const void*)prefill_attn_pp_kernel, smem)) return rc;
    const int grid = a.units < host_sm_count() ? a.units : host_sm_count();
    return launch_kernel((const void*)prefill_attn_pp_kernel, dim3(grid), dim3(kPpThreads), smem, 1, stream, &a);
  }
  const int smem = PaLayout::total;
  if (int rc = set_max_dynamic_smem((const void*)prefill_attn_kernel, smem)) return rc;
  const int grid = units < host_sm_count() ? (int)units : host_sm_count();
  return launch_kernel((const void*)prefill_attn_kernel, dim3(grid), dim3(kPaThreads), smem, 1, stream, &a);
}
