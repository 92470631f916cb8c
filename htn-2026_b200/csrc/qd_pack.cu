// Weight packing (load time) and the embedding gather (first op of every decode step).
#include "qd_common.cuh"
#include "qd_host.h"

namespace qd {

struct PackArgs {
  const uint4* src;
  int64_t ld_src8;  // source row stride in 16-byte chunks
  int64_t n_src, k8, kblocks;
  int64_t span, group_stride, row_offset;
  __nv_bfloat16* dst;
};

__global__ void pack_rows_kernel(const __grid_constant__ PackArgs a) {
  const int64_t total = a.n_src * a.k8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = i / a.k8, q = i - j * a.k8;
    const int64_t row = (j / a.span) * a.group_stride + a.row_offset + (j % a.span);
    const uint4 v = a.src[j * a.ld_src8 + q];
    *reinterpret_cast<uint4*>(a.dst + packed_offset_elems(row, q * 8, a.kblocks)) = v;
  }
}

struct EmbedArgs {
  const int64_t* tok;
  const __nv_bfloat16* e;
  int64_t vocab, k8, kblocks;
  __nv_bfloat16* x;
  int64_t ldx;
  int* err;
};

__global__ void embed_kernel(const __grid_constant__ EmbedArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int i = blockIdx.x;
  int64_t t = ld_cg_s64(a.tok + i);
  if (t < 0 || t >= a.vocab) {
    if (threadIdx.x == 0 && a.err) atomicOr(a.err, QD_DEVERR_TOKEN);
    t = t < 0 ? 0 : a.vocab - 1;
  }
  for (int64_t q = threadIdx.x; q < a.k8; q += blockDim.x) {
    const uint4 v = *reinterpret_cast<const uint4*>(a.e + packed_offset_elems(t, q * 8, a.kblocks));
    *reinterpret_cast<uint4*>(a.x + i * a.ldx + q * 8) = v;
  }
}

}  // namespace qd

using namespace qd;

extern "C" int64_t qd_packed_bytes(int64_t n_rows, int64_t k) {
  if (n_rows <= 0 || k <= 0) return 0;
  return (n_rows + kBlockRows - 1) / kBlockRows * kBlockRows * ((k + kBlockCols - 1) / kBlockCols * kBlockCols) * 2;
}

extern "C" int qd_pack_rows(const void* src, int64_t ld_src, int64_t n_src_rows, int64_t k, void* dst,
                            int64_t n_dst_rows, int64_t span, int64_t group_stride, int64_t row_offset,
                            cudaStream_t stream) {
  if (!src || !dst) return set_error(QD_ERR_ARG, "null pointer");
  if (n_src_rows <= 0 || k <= 0 || k % kBlockCols || n_dst_rows % kBlockRows || span <= 0 || row_offset < 0 ||
      group_stride < 0)
    return set_error(QD_ERR_ARG, "pack: bad sizes (k%%64, n_dst%%128, span>0)");
  if (!aligned16(src) || !aligned16(dst) || ld_src < k || ld_src % 8)
    return set_error(QD_ERR_ARG, "pack: src/dst 16-byte aligned, ld_src >= k and a multiple of 8");
  // either plain stacking (one span covers every row) or interleaving with non-overlapping groups;
  // in both cases the last source row maps to the largest destination row
  const bool plain = group_stride == 0 && span >= n_src_rows;
  if (!plain && group_stride < span) return set_error(QD_ERR_ARG, "pack: group_stride < span would overlap rows");
  const int64_t last = ((n_src_rows - 1) / span) * group_stride + row_offset + (n_src_rows - 1) % span;
  if (last >= n_dst_rows) return set_error(QD_ERR_ARG, "pack: rows map outside the destination");
  PackArgs a;
  a.src = static_cast<const uint4*>(src);
  a.ld_src8 = ld_src / 8;
  a.n_src = n_src_rows;
  a.k8 = k / 8;
  a.kblocks = k / kBlockCols;
  a.span = span;
  a.group_stride = group_stride;
  a.row_offset = row_offset;
  a.dst = static_cast<__nv_bfloat16*>(dst);
  const int64_t total = n_src_rows * a.k8;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 65535 * 8) blocks = 65535 * 8;
  return launch_kernel((const void*)pack_rows_kernel, dim3(blocks), dim3(256), 0, 0, stream, &a);
}

extern "C" int qd_embed(const int64_t* tok, const void* e_packed, int64_t vocab, int64_t k, int m, void* x,
                        int64_t ldx, int* err, int pdl, cudaStream_t stream) {
  if (!tok || !e_packed || !x) return set_error(QD_ERR_ARG, "null pointer");
  if (m < 1 || vocab <= 0 || k <= 0 || k % kBlockCols || ldx < k || ldx % 8 || !aligned16(x) || !aligned16(e_packed))
    return set_error(QD_ERR_ARG, "embed: bad sizes or alignment");
  EmbedArgs a;
  a.tok = tok;
  a.e = static_cast<const __nv_bfloat16*>(e_packed);
  a.vocab = vocab;
  a.k8 = k / 8;
  a.kblocks = k / kBlockCols;
  a.x = static_cast<__nv_bfloat16*>(x);
  a.ldx = ldx;
  a.err = err;
  return launch_kernel((const void*)embed_kernel, dim3(m), dim3(128), 0, pdl, stream, &a);
}
