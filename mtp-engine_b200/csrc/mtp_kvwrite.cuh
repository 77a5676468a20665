// mtp_kvwrite.cuh -- batched write of new K/V rows into the PagedKVCache page
// pool, replacing the per-token PagedKVCache.write_inplace
// (mtp_engine.py:582-586), which reads each page id back to the host.
//
// Row (b, h, t), t < n (and t < count[b] when counts are given):
//   logical = start + t, page = page_table[b, logical], slot = logical % page_size
//   k_pages[page, b, h, slot, :] = src_k[b, h, node(b, t), :]   (v likewise)
// with node(b, t) = node_idx[b, t] (e.g. the accepted path of a draft tree)
// or t.  One warp per row; 16-byte chunks when source and pool share a dtype
// and both are aligned, else element by element with conversion (the
// reference casts with .to(self.dtype), line 584).  Page ids resolve like the
// reference's integer indexing (resolve_page: -1 selects the last page); an
// id outside [-P, P) or a node index outside the source skips the row and
// records MTP_ERR_DEVICE.  When several tokens of one call map to the same
// (page, slot), the last of them is written, as in the reference's loop.
#pragma once

#include "mtp_common.cuh"

namespace mtp {

struct KvWriteArgs {
  void* k_pages;
  void* v_pages;
  int dtype;  // pool dtype
  const int32_t* page_table;
  int64_t table_stride, num_pages, page_size;
  const void* src_k;
  const void* src_v;
  int src_dtype;
  int64_t src_len;
  const int32_t* node_idx;  // [B, n] or null
  const int32_t* count;     // [B] or null
  int64_t B, H, D, start, n;
  int vec;  // 16-byte chunks
};

__global__ void __launch_bounds__(256) paged_kv_write_kernel(KvWriteArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);  // (b, h, t), t fastest
  if (row >= a.B * a.H * a.n) return;
  const int64_t t = row % a.n;
  const int64_t h = (row / a.n) % a.H;
  const int64_t b = row / (a.n * a.H);
  if (a.count && t >= (int64_t)a.count[b]) return;
  const int64_t logical = a.start + t;
  const int64_t page = resolve_page(a.page_table[b * a.table_stride + logical], a.num_pages);
  const int64_t node = a.node_idx ? (int64_t)a.node_idx[b * a.n + t] : t;
  if (page < 0 || node < 0 || node >= a.src_len) {
    if (lane == 0) record_error(MTP_ERR_DEVICE);
    return;
  }
  // The reference writes token after token, so when two tokens of this call
  // land on one (page, slot) -- a -1 column aliasing page P-1, or a table
  // that maps two pages' slots to one page -- the later token stays.  Tokens
  // t < t2 share a slot only if t2 - t is a multiple of page_size: the lanes
  // check t + page_size, t + 2 page_size, ... and this row yields if any of
  // them (within its sequence's count) resolves to the same page.
  const int64_t nb = a.count ? min(a.n, (int64_t)a.count[b]) : a.n;
  bool later = false;
  for (int64_t t2 = t + (int64_t)(lane + 1) * a.page_size; t2 < nb; t2 += 32 * a.page_size)
    later |= resolve_page(a.page_table[b * a.table_stride + a.start + t2], a.num_pages) == page;
  if (__any_sync(0xffffffffu, later)) return;
  const int64_t dst = ((((int64_t)page * a.B + b) * a.H + h) * a.page_size + logical % a.page_size) * a.D;
  const int64_t src = ((b * a.H + h) * a.src_len + node) * a.D;
  if (a.vec) {
    const int eb = a.dtype == MTP_DTYPE_F32 ? 4 : 2;
    const int64_t chunks = a.D * eb / 16;
    const uint4* sk = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.src_k) + src * eb);
    const uint4* sv = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.src_v) + src * eb);
    uint4* dk = reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.k_pages) + dst * eb);
    uint4* dv = reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.v_pages) + dst * eb);
    for (int64_t c = lane; c < chunks; c += 32) {
      dk[c] = __ldg(sk + c);
      dv[c] = __ldg(sv + c);
    }
  } else {
    for (int64_t d = lane; d < a.D; d += 32) {
      store_f32(a.k_pages, a.dtype, dst + d, load_f32(a.src_k, a.src_dtype, src + d));
      store_f32(a.v_pages, a.dtype, dst + d, load_f32(a.src_v, a.src_dtype, src + d));
    }
  }
}

}  // namespace mtp
