// Host-side plans shared by the per-projection kernels and the persistent decode-step kernel.
#pragma once

#include <stdint.h>

namespace qd {

// Stream-K GEMV plan over a packed [n_rows, k] matrix for m activation rows.
struct Plan {
  int grid, smax, nst;
  int64_t groups, total;
  int64_t off_tickets, off_lm_ticket, off_cta_val, off_cta_idx, off_partials, bytes;
};
bool make_plan(int64_t n_rows, int64_t k, int M, int grid_hint, Plan* p);
// Largest number of CTAs that share one row group under the stream-K split of groups x kblocks blocks.
int stream_k_smax(int64_t groups, int kblocks, int grid);

// Split-K attention plan: splits x chunk covers the cache capacity.
struct AttnPlan {
  int splits;
  int64_t chunk, off_acc, off_ml, off_tickets, bytes;
};
bool attn_plan(int batch, int nkv, int64_t cap, int grid_hint, AttnPlan* p);

int env_int(const char* name, int dflt);
// Keys per attention split at run time.
int attn_keys_per_split();
// Blocks each CTA keeps prefetched into L2 beyond its shared-memory ring.
int prefetch_blocks();

}  // namespace qd
