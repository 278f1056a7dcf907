// Sliding-window cache as a ring over a sequence's pool blocks: the host
// state of RotatingKVCache (crates/rmlx-serve-cache/src/rotating_cache.rs:
// 16-283) behind the C ABI.
//
// The reference keeps max_size rows per (layer, head) in a Vec and moves
// `written` and `offset` as tokens arrive.  Here the rows live in the paged
// pool: ring position p is row p % block_size of block table entry
// p / block_size, and blocks are taken from the block manager as the ring
// first reaches them (the reference preallocates max_size rows).  This
// object turns the reference's bookkeeping into the device calls:
//   append (:94-143)        -> the slot of each new token (rmlx_kv_append);
//   get_logical_order       -> the ring offset rmlx_kv_gather_ring takes;
//     (:162-197)
//   trim (:213-247)         -> before the ring rotates, the row shift as
//                              (src, dst) slot pairs for rmlx_kv_move_rows;
//                              after, only the offset moves;
//   seq_len / can_trim      -> the same formulas (:201-203, :253-255).
// The state advances once per token for all of a pool's layers; the
// reference advances it on each per-layer append call, which is the same for
// a one-layer cache and for each layer driven as its own cache.
#include <new>
#include <vector>

#include "block_manager.h"

using rmlx::fail;

struct rmlx_rotating {
  rmlx::BlockManager* mgr;
  int64_t bs, max_size, keep;
  int64_t offset = 0, written = 0;
  std::vector<int32_t> table;
  std::vector<int32_t> last;  // append_slots: the token that last took each ring position (-1: none)

  int64_t rotating() const { return max_size - keep; }
  int64_t seq_len() const { return written < max_size ? written : max_size; }
  // Ring position of the next token, as append computes write_pos (:121-127).
  int64_t next_pos(int64_t w, int64_t off) const { return w < max_size ? w : keep + off; }
  int32_t slot(int64_t pos) const { return (int32_t)(table[pos / bs] * bs + pos % bs); }
};

extern "C" {

rmlx_status rmlx_rotating_new(rmlx_block_manager* m, int32_t block_size, int32_t max_size, int32_t keep,
                              rmlx_rotating** out) {
  if (!m || !out) return fail(RMLX_E_BAD_ARG, "NULL manager or out");
  *out = nullptr;
  if (block_size <= 0 || (size_t)block_size != m->impl.block_size())
    return fail(RMLX_E_BAD_ARG, "block_size %d differs from the manager's %zu", block_size, m->impl.block_size());
  if (keep < 0 || max_size <= 0) return fail(RMLX_E_BAD_ARG, "max_size must be > 0 and keep >= 0");
  if (keep >= max_size)  // rotating_cache.rs:53-56
    return fail(RMLX_E_BAD_ARG, "keep (%d) must be less than max_size (%d)", keep, max_size);
  rmlx_rotating* r = new (std::nothrow) rmlx_rotating();
  if (!r) return fail(RMLX_E_EXHAUSTED, "host allocation failed");
  r->mgr = &m->impl;
  r->bs = block_size;
  r->max_size = max_size;
  r->keep = keep;
  *out = r;
  return RMLX_OK;
}

void rmlx_rotating_release(rmlx_rotating* r) {
  if (!r) return;
  for (int32_t b : r->table) r->mgr->free_block(b);
  r->table.clear();
  r->written = r->offset = 0;
}

void rmlx_rotating_destroy(rmlx_rotating* r) {
  rmlx_rotating_release(r);
  delete r;
}

rmlx_status rmlx_rotating_append_slots(rmlx_rotating* r, int32_t n, int32_t* slots) {
  if (!r) return fail(RMLX_E_BAD_ARG, "NULL ring");
  if (n < 0) return fail(RMLX_E_BAD_ARG, "n < 0");
  if (n == 0) return RMLX_OK;
  if (!slots) return fail(RMLX_E_BAD_ARG, "NULL slots");
  // The highest ring position the n tokens reach: the blocks up to it are
  // taken first, so that an exhausted pool leaves the state unchanged.
  int64_t w = r->written, off = r->offset, top = -1;
  for (int32_t t = 0; t < n; ++t) {
    const int64_t pos = r->next_pos(w, off);
    if (pos > top) top = pos;
    if (w >= r->max_size) off = (off + 1) % r->rotating();
    ++w;
    if (w >= r->max_size && top >= r->max_size - 1) break;  // every position reached
  }
  const size_t need = (size_t)(top / r->bs + 1);
  if (need > r->table.size()) {
    if (need - r->table.size() > r->mgr->num_free())
      return fail(RMLX_E_EXHAUSTED, "ring needs %zu more blocks, %zu free", need - r->table.size(),
                  r->mgr->num_free());
    while (r->table.size() < need) {
      int32_t b;
      r->mgr->allocate(&b);
      r->table.push_back(b);
    }
  }
  // A position written twice within the call keeps the later token; the
  // earlier one's slot is -1, which rmlx_kv_append skips.  A call can revisit
  // a position only when it has more tokens than the ring rotates through,
  // or when a trim of a rotated ring left written < max_size with a nonzero
  // offset (the linear fill then runs into the rotating positions).
  const bool revisit =
      n > 1 && ((int64_t)n > r->rotating() || (r->written < r->max_size && r->offset != 0));
  if (revisit && r->last.size() != (size_t)r->max_size) r->last.assign((size_t)r->max_size, -1);
  const int64_t w0 = r->written, off0 = r->offset;
  for (int32_t t = 0; t < n; ++t) {
    const int64_t pos = r->next_pos(r->written, r->offset);
    slots[t] = r->slot(pos);
    if (revisit) {
      if (r->last[pos] >= 0) slots[r->last[pos]] = -1;
      r->last[pos] = t;
    }
    if (r->written >= r->max_size) r->offset = (r->offset + 1) % r->rotating();
    ++r->written;
  }
  if (revisit) {  // leave the scratch all -1 for the next call
    int64_t w = w0, off = off0;
    for (int32_t t = 0; t < n; ++t) {
      r->last[r->next_pos(w, off)] = -1;
      if (w >= r->max_size) off = (off + 1) % r->rotating();
      ++w;
    }
  }
  return RMLX_OK;
}

size_t rmlx_rotating_seq_len(const rmlx_rotating* r) { return r ? (size_t)r->seq_len() : 0; }
int32_t rmlx_rotating_can_trim(const rmlx_rotating* r) { return r && r->seq_len() > r->keep; }
int32_t rmlx_rotating_ring_offset(const rmlx_rotating* r) {
  return !r || r->written <= r->max_size ? -1 : (int32_t)r->offset;
}
size_t rmlx_rotating_written(const rmlx_rotating* r) { return r ? (size_t)r->written : 0; }
size_t rmlx_rotating_max_size(const rmlx_rotating* r) { return r ? (size_t)r->max_size : 0; }
size_t rmlx_rotating_keep(const rmlx_rotating* r) { return r ? (size_t)r->keep : 0; }

rmlx_status rmlx_rotating_trim(rmlx_rotating* r, int32_t n, int32_t* src_slots, int32_t* dst_slots, int32_t cap,
                               int32_t* n_moves) {
  if (!r || !n_moves) return fail(RMLX_E_BAD_ARG, "NULL ring or n_moves");
  *n_moves = 0;
  if (n < 0) return fail(RMLX_E_BAD_ARG, "n < 0");
  const int64_t trimmable = r->seq_len() > r->keep ? r->seq_len() - r->keep : 0;
  if (n > trimmable)  // rotating_cache.rs:215-219
    return fail(RMLX_E_RANGE, "cannot trim %d tokens: only %lld trimmable", n, (long long)trimmable);
  if (r->written <= r->max_size) {
    // Not rotating: rows [keep + n, written) move down by n (:221-238).
    const int64_t remaining = r->written - r->keep - n;
    *n_moves = (int32_t)remaining;
    if (remaining > 0 && (cap < remaining || !src_slots || !dst_slots))
      return fail(RMLX_E_BAD_ARG, "trim moves %lld rows, room for %d", (long long)remaining, cap);
    for (int64_t i = 0; i < remaining; ++i) {
      src_slots[i] = r->slot(r->keep + n + i);
      dst_slots[i] = r->slot(r->keep + i);
    }
    r->written -= n;
  } else {
    // Rotating: the oldest rows are skipped by the offset (:239-246).
    r->offset = (r->offset + n) % r->rotating();
    r->written -= n;
  }
  return RMLX_OK;
}

rmlx_status rmlx_rotating_blocks(const rmlx_rotating* r, int32_t* out, int32_t cap, int32_t* n_blocks) {
  if (!r || !n_blocks) return fail(RMLX_E_BAD_ARG, "NULL ring or n_blocks");
  *n_blocks = (int32_t)r->table.size();
  if (!out) return RMLX_OK;
  if ((size_t)cap < r->table.size()) return fail(RMLX_E_BAD_ARG, "room for %d blocks, %zu held", cap, r->table.size());
  for (size_t i = 0; i < r->table.size(); ++i) out[i] = r->table[i];
  return RMLX_OK;
}

}  // extern "C"
