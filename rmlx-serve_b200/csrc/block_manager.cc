// Host-side paged block manager: the drop-in for PagedCacheManager
// (crates/rmlx-serve-cache/src/paged_cache.rs:71-302).
//
// Same observable behaviour as the reference -- FIFO reuse of freed blocks,
// reference counts, copy-on-write metadata, and a content-hash index whose
// entries survive append_tokens (paged_cache.rs:299-300) and are removed on
// free only when they still point at the freed block (:139-145) -- with a
// layout chosen for a scheduler that touches thousands of blocks per step:
//   * the free list is a fixed ring of int32 ids (no per-op allocation);
//   * per-block state is struct-of-arrays, token ids live in one flat
//     [num_blocks][block_size] array (tokens.len() == num_filled always);
//   * the hash index is an open-addressing map (FlatMap64).
#include <cstdarg>
#include <cstdlib>
#include <new>

#include "block_manager.h"

namespace rmlx {

static thread_local std::string g_last_error;

rmlx_status fail(rmlx_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}
void clear_error() { g_last_error.clear(); }
const char* last_error() { return g_last_error.c_str(); }

}  // namespace rmlx

using rmlx::BlockManager;
using rmlx::fail;


extern "C" {

const char* rmlx_last_error(void) { return rmlx::last_error(); }

const char* rmlx_version(void) { return "0.1.0"; }

const char* rmlx_status_string(rmlx_status s) {
  switch (s) {
    case RMLX_OK: return "ok";
    case RMLX_E_RANGE: return "block id out of range";
    case RMLX_E_DOUBLE_FREE: return "double free";
    case RMLX_E_OVERFLOW: return "block overflow";
    case RMLX_E_FREE_BLOCK: return "block is free";
    case RMLX_E_BAD_ARG: return "bad argument";
    case RMLX_E_EXHAUSTED: return "exhausted";
    case RMLX_E_CUDA: return "cuda error";
    case RMLX_E_NCCL: return "nccl error";
    case RMLX_E_TIMEOUT: return "timeout";
    case RMLX_E_DEVICE: return "device-side validation error";
  }
  return "unknown status";
}

rmlx_status rmlx_block_manager_new(size_t block_size, size_t num_blocks, rmlx_block_manager** out) {
  if (!out) return fail(RMLX_E_BAD_ARG, "out is NULL");
  if (block_size == 0) return fail(RMLX_E_BAD_ARG, "block_size must be > 0");
  if (num_blocks > (size_t)INT32_MAX) return fail(RMLX_E_BAD_ARG, "num_blocks exceeds int32 ids");
  *out = new (std::nothrow) rmlx_block_manager(block_size, num_blocks);
  return *out ? RMLX_OK : fail(RMLX_E_EXHAUSTED, "host allocation failed");
}
void rmlx_block_manager_destroy(rmlx_block_manager* m) { delete m; }

rmlx_status rmlx_block_manager_allocate(rmlx_block_manager* m, int32_t* id, int32_t* found) {
  *found = m->impl.allocate(id) ? 1 : 0;
  return RMLX_OK;
}
rmlx_status rmlx_block_manager_allocate_n(rmlx_block_manager* m, size_t n, int32_t* ids, size_t* n_got) {
  size_t i = 0;
  while (i < n && m->impl.allocate(&ids[i])) ++i;
  *n_got = i;
  return RMLX_OK;
}
rmlx_status rmlx_block_manager_free(rmlx_block_manager* m, int32_t id) { return m->impl.free_block(id); }
rmlx_status rmlx_block_manager_free_n(rmlx_block_manager* m, const int32_t* ids, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    rmlx_status s = m->impl.free_block(ids[i]);
    if (s != RMLX_OK) return s;
  }
  return RMLX_OK;
}
rmlx_status rmlx_block_manager_ref_count(const rmlx_block_manager* m, int32_t id, size_t* out) {
  return m->impl.ref_count(id, out);
}
rmlx_status rmlx_block_manager_increment_ref(rmlx_block_manager* m, int32_t id) { return m->impl.increment_ref(id); }
rmlx_status rmlx_block_manager_copy_on_write(rmlx_block_manager* m, int32_t id, int32_t* nid, int32_t* copied) {
  return m->impl.copy_on_write(id, nid, copied);
}
size_t rmlx_block_manager_num_free_blocks(const rmlx_block_manager* m) { return m->impl.num_free(); }
size_t rmlx_block_manager_num_allocated_blocks(const rmlx_block_manager* m) {
  return m->impl.num_blocks() - m->impl.num_free();
}
size_t rmlx_block_manager_num_blocks(const rmlx_block_manager* m) { return m->impl.num_blocks(); }
size_t rmlx_block_manager_block_size(const rmlx_block_manager* m) { return m->impl.block_size(); }
rmlx_status rmlx_block_manager_get_block(const rmlx_block_manager* m, int32_t id, rmlx_block_view* v,
                                         uint32_t* tokens, size_t cap, int32_t* found) {
  *found = m->impl.view(id, v, tokens, tokens ? cap : 0) ? 1 : 0;
  return RMLX_OK;
}
rmlx_status rmlx_block_manager_register_hash(rmlx_block_manager* m, int32_t id, uint64_t h) {
  return m->impl.register_hash(id, h);
}
rmlx_status rmlx_block_manager_lookup_hash(const rmlx_block_manager* m, uint64_t h, int32_t* id, int32_t* found) {
  *found = m->impl.lookup_hash(h, id) ? 1 : 0;
  return RMLX_OK;
}
rmlx_status rmlx_block_manager_append_tokens(rmlx_block_manager* m, int32_t id, const uint32_t* t, size_t n) {
  return m->impl.append_tokens(id, t, n);
}

}  // extern "C"
