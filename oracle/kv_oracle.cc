// ORACLE -- TEST INFRASTRUCTURE ONLY.
//
// A single-threaded CPU restatement of rmlx-serve's KV-cache crate
// (crates/rmlx-serve-cache/src/*.rs, Rust) used as the parity checker for the
// CUDA path in rmlx-serve_b200/.  Only tests/, __graft_entry__.smoke() and the
// CPU-baseline leg of bench.py load this library; the product never links,
// calls or ships it.
//
// Every function cites the reference line range it restates.  Arithmetic
// follows the Rust semantics exactly: f32 division, `f32::max/min` folds
// (fmaxf/fminf), `round()` = roundf (half away from zero), saturating `as u8`,
// and multiply-then-add dequantisation (built with -ffp-contract=off so that
// nothing is fused into an FMA).
//
// Pieces with no reference implementation are build-defined and say so:
//   * paged K/V data append/gather/copy: the reference's only value-moving
//     append/gather is RotatingKVCache (rotating_cache.rs:94-197); the paged
//     variant below keeps its per-head row copy semantics and adds the block
//     table mapping (slot = block * block_size + offset).
//   * prefix-block chain hash: the reference takes caller-supplied hashes
//     (paged_cache.rs:265-272) and computes none.  The chain hash here is
//     XXH64 (Yann Collet's published algorithm, seed 0) over
//     le64(parent_hash) || le32(token ids of the block).
//
// Panicking reference paths (assert!) return a nonzero status instead.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <deque>
#include <thread>
#include <unordered_map>
#include <vector>

extern "C" {
enum {
  ORC_OK = 0,
  ORC_E_RANGE = 1,        // block id out of range (paged_cache.rs:126-130)
  ORC_E_DOUBLE_FREE = 2,  // free of a block with ref_count 0 (:132-135)
  ORC_E_OVERFLOW = 3,     // append_tokens overflow (:290-296)
  ORC_E_FREE_BLOCK = 4,   // increment_ref on a free block (:177-180)
  ORC_E_BAD_ARG = 5,      // bits not 4/8, length mismatch, slice panic
};
}

namespace orc {

// ---------------------------------------------------------------------------
// PagedCacheManager -- paged_cache.rs:14-301
// ---------------------------------------------------------------------------
struct Block {  // KVCacheBlock, paged_cache.rs:14-26
  size_t block_id = 0;
  size_t ref_count = 0;
  bool has_hash = false;
  uint64_t hash = 0;
  std::vector<uint32_t> tokens;
  size_t num_filled = 0;
  void reset() {  // :51-56
    ref_count = 0;
    has_hash = false;
    hash = 0;
    tokens.clear();
    num_filled = 0;
  }
};

struct PagedManager {
  size_t block_size, num_blocks;
  std::deque<size_t> free_blocks;
  std::vector<Block> blocks;
  std::unordered_map<uint64_t, size_t> hash_to_block;

  PagedManager(size_t bs, size_t n) : block_size(bs), num_blocks(n), blocks(n) {  // :90-104
    for (size_t i = 0; i < n; ++i) {
      blocks[i].block_id = i;
      free_blocks.push_back(i);
    }
  }
  bool allocate(size_t* out) {  // :110-115
    if (free_blocks.empty()) return false;
    size_t id = free_blocks.front();
    free_blocks.pop_front();
    blocks[id].reset();
    blocks[id].ref_count = 1;
    *out = id;
    return true;
  }
  int free_block(size_t id) {  // :125-149
    if (id >= num_blocks) return ORC_E_RANGE;
    Block& b = blocks[id];
    if (b.ref_count == 0) return ORC_E_DOUBLE_FREE;
    b.ref_count -= 1;
    if (b.ref_count == 0) {
      if (b.has_hash) {
        auto it = hash_to_block.find(b.hash);
        if (it != hash_to_block.end() && it->second == id) hash_to_block.erase(it);
      }
      b.reset();
      free_blocks.push_back(id);
    }
    return ORC_OK;
  }
  int ref_count(size_t id, size_t* out) const {  // :157-163
    if (id >= num_blocks) return ORC_E_RANGE;
    *out = blocks[id].ref_count;
    return ORC_OK;
  }
  int increment_ref(size_t id) {  // :172-182
    if (id >= num_blocks) return ORC_E_RANGE;
    if (blocks[id].ref_count == 0) return ORC_E_FREE_BLOCK;
    blocks[id].ref_count += 1;
    return ORC_OK;
  }
  // :197-224.  Returns ORC_OK with *copied=0 for the reference's None.
  int copy_on_write(size_t id, size_t* out, int* copied) {
    *copied = 0;
    if (id >= num_blocks) return ORC_E_RANGE;
    if (blocks[id].ref_count <= 1) return ORC_OK;
    size_t nid;
    if (!allocate(&nid)) return ORC_OK;
    blocks[nid].tokens = blocks[id].tokens;
    blocks[nid].num_filled = blocks[id].num_filled;
    blocks[nid].has_hash = false;
    blocks[id].ref_count -= 1;
    *out = nid;
    *copied = 1;
    return ORC_OK;
  }
  int register_hash(size_t id, uint64_t h) {  // :265-272
    if (id >= num_blocks) return ORC_E_RANGE;
    blocks[id].has_hash = true;
    blocks[id].hash = h;
    hash_to_block[h] = id;
    return ORC_OK;
  }
  bool lookup_hash(uint64_t h, size_t* out) const {  // :278-282
    auto it = hash_to_block.find(h);
    if (it == hash_to_block.end()) return false;
    if (blocks[it->second].ref_count == 0) return false;
    *out = it->second;
    return true;
  }
  int append_tokens(size_t id, const uint32_t* t, size_t n) {  // :288-301
    if (id >= num_blocks) return ORC_E_RANGE;  // Rust indexing panic
    Block& b = blocks[id];
    if (b.num_filled + n > block_size) return ORC_E_OVERFLOW;
    b.tokens.insert(b.tokens.end(), t, t + n);
    b.num_filled += n;
    b.has_hash = false;
    return ORC_OK;
  }
};

// ---------------------------------------------------------------------------
// PrefixCacheManager -- prefix_cache.rs:14-291
// ---------------------------------------------------------------------------
struct TrieNode {  // :14-22
  std::unordered_map<uint32_t, size_t> children;
  bool has_block = false;
  size_t block_id = 0;
  uint64_t last_access = 0;
};

struct PrefixCache {
  std::vector<TrieNode> nodes;
  uint64_t access_counter = 0;
  size_t max_blocks;
  size_t num_blocks = 0;
  uint64_t total_lookups = 0, hit_tokens = 0, lookup_tokens = 0;

  explicit PrefixCache(size_t maxb) : nodes(1), max_blocks(maxb) {}  // :66-77

  std::vector<size_t> lookup(const uint32_t* tokens, size_t n) {  // :85-113
    total_lookups += 1;
    lookup_tokens += n;
    std::vector<size_t> ids;
    size_t cur = 0;
    access_counter += 1;
    uint64_t t = access_counter;
    for (size_t i = 0; i < n; ++i) {
      auto it = nodes[cur].children.find(tokens[i]);
      if (it == nodes[cur].children.end()) break;
      cur = it->second;
      nodes[cur].last_access = t;
      if (nodes[cur].has_block) ids.push_back(nodes[cur].block_id);
    }
    hit_tokens += ids.size();
    return ids;
  }

  void insert(const uint32_t* tokens, size_t n, const size_t* ids, size_t nb) {  // :126-179
    insert_report(tokens, n, ids, nb, nullptr, nullptr);
  }
  // insert (:126-179) that also records, per block index, whether the
  // boundary node had no block (attached) and the block it replaced.
  void insert_report(const uint32_t* tokens, size_t n, const size_t* ids, size_t nb, std::vector<int>* attached,
                     std::vector<long long>* replaced) {
    if (attached) attached->assign(nb, 0);
    if (replaced) replaced->assign(nb, -1);
    if (n == 0 || nb == 0) return;
    size_t tpb = (nb == 1) ? n : n / nb;
    access_counter += 1;
    uint64_t t = access_counter;
    size_t cur = 0, bi = 0;
    for (size_t i = 0; i < n; ++i) {
      size_t next;
      auto it = nodes[cur].children.find(tokens[i]);
      if (it != nodes[cur].children.end()) {
        next = it->second;
      } else {
        next = nodes.size();
        nodes.emplace_back();
        nodes[cur].children[tokens[i]] = next;
      }
      nodes[next].last_access = t;
      bool boundary = false;
      if (bi < nb) {
        if (bi == nb - 1) boundary = (i == n - 1);
        else boundary = (i + 1) == (bi + 1) * tpb;
      }
      if (boundary && bi < nb) {
        bool had = nodes[next].has_block;
        if (had && replaced && nodes[next].block_id != ids[bi]) (*replaced)[bi] = (long long)nodes[next].block_id;
        nodes[next].has_block = true;
        nodes[next].block_id = ids[bi];
        if (!had) num_blocks += 1;
        if (!had && attached) (*attached)[bi] = 1;
        bi += 1;
      }
      cur = next;
    }
  }

  bool evict_lru(size_t* out) {  // :187-232
    if (num_blocks == 0) return false;
    bool found = false;
    size_t best = 0;
    uint64_t best_access = UINT64_MAX;
    bool best_leaf = false;
    for (size_t idx = 0; idx < nodes.size(); ++idx) {
      const TrieNode& nd = nodes[idx];
      if (!nd.has_block) continue;
      bool leaf = nd.children.empty();
      bool better;
      if (leaf && !best_leaf) better = true;
      else if (!leaf && best_leaf) better = false;
      else better = nd.last_access < best_access;
      if (better) {
        found = true;
        best = idx;
        best_access = nd.last_access;
        best_leaf = leaf;
      }
    }
    if (!found) return false;
    *out = nodes[best].block_id;
    nodes[best].has_block = false;
    num_blocks -= 1;
    if (best_leaf) prune_leaf(best);
    return true;
  }

  void prune_leaf(size_t leaf) {  // :235-260
    if (leaf == 0) return;
    if (!nodes[leaf].children.empty() || nodes[leaf].has_block) return;
    for (size_t p = 0; p < nodes.size(); ++p) {
      auto& ch = nodes[p].children;
      for (auto it = ch.begin(); it != ch.end(); ++it) {
        if (it->second == leaf) {
          ch.erase(it);
          return;
        }
      }
    }
  }

  double hit_rate() const {  // :266-271
    if (lookup_tokens == 0) return 0.0;
    return (double)hit_tokens / (double)lookup_tokens;
  }
};

// ---------------------------------------------------------------------------
// MemoryAwarePrefixCache -- memory.rs:10-158 (Linux: available_memory_mb()
// returns usize::MAX, memory.rs:88-91)
// ---------------------------------------------------------------------------
struct MemPrefix {
  PrefixCache pc;
  size_t limit, usage = 0, bpb;
  std::vector<size_t> evicted_log;  // block ids dropped by eviction, in order
  MemPrefix(size_t maxb, size_t limit_mb, size_t bpb_) : pc(maxb), limit(limit_mb * 1024 * 1024), bpb(bpb_) {}
  bool should_evict() const {  // :99-110
    if (usage >= limit) return true;
    if (pc.num_blocks >= pc.max_blocks) return true;
    size_t avail = SIZE_MAX;
    size_t thr = limit / (1024 * 1024) / 10;
    return avail < (thr > 256 ? thr : 256);
  }
  void evict_until_threshold() {  // :117-136
    size_t target = (size_t)((double)limit * 0.8);
    while (usage > target) {
      size_t id;
      if (pc.evict_lru(&id)) {
        usage = usage > bpb ? usage - bpb : 0;
        evicted_log.push_back(id);
      } else {
        break;
      }
    }
  }
  void insert(const uint32_t* t, size_t n, const size_t* ids, size_t nb) {  // :149-158
    if (should_evict()) evict_until_threshold();
    pc.insert(t, n, ids, nb);
    usage += nb * bpb;
  }
  bool evict_lru(size_t* out) {  // :161-168
    bool ok = pc.evict_lru(out);
    if (ok) usage = usage > bpb ? usage - bpb : 0;
    return ok;
  }
};

// ---------------------------------------------------------------------------
// QuantizedKVCache group math -- quantized_cache.rs:177-296
// ---------------------------------------------------------------------------
static inline uint8_t sat_u8(float x) {  // Rust `as u8` after clamp: NaN -> 0
  if (x != x) return 0;
  if (x <= 0.0f) return 0;
  if (x >= 255.0f) return 255;
  return (uint8_t)x;
}
static inline float clampq(float x, float qmax) {  // f32::clamp(0.0, qmax)
  if (x < 0.0f) return 0.0f;
  if (x > qmax) return qmax;
  return x;
}

// quantize_group, :232-273.  Appends packed bytes to `out`.
static void quantize_group(const float* d, size_t n, int bits, std::vector<uint8_t>& out,
                           float* scale_out, float* zero_out) {
  if (n == 0) {
    *scale_out = 0.0f;
    *zero_out = 0.0f;
    return;
  }
  float mx = -INFINITY, mn = INFINITY;
  for (size_t i = 0; i < n; ++i) mx = fmaxf(mx, d[i]);
  for (size_t i = 0; i < n; ++i) mn = fminf(mn, d[i]);
  float qmax = (float)((1u << bits) - 1);
  float range = mx - mn;
  float scale = (range == 0.0f) ? 1.0f : range / qmax;
  if (bits == 8) {
    for (size_t i = 0; i < n; ++i) out.push_back(sat_u8(clampq(roundf((d[i] - mn) / scale), qmax)));
  } else {
    for (size_t i = 0; i < n; i += 2) {
      uint8_t lo = sat_u8(clampq(roundf((d[i] - mn) / scale), qmax));
      uint8_t hi = (i + 1 < n) ? sat_u8(clampq(roundf((d[i + 1] - mn) / scale), qmax)) : 0;
      out.push_back((uint8_t)(lo | (hi << 4)));
    }
  }
  *scale_out = scale;
  *zero_out = mn;
}

// dequantize_group, :278-296
static void dequantize_group(const uint8_t* b, size_t nb, float scale, float zero, int bits,
                             std::vector<float>& out) {
  if (bits == 8) {
    for (size_t i = 0; i < nb; ++i) out.push_back((float)b[i] * scale + zero);
  } else {
    for (size_t i = 0; i < nb; ++i) {
      float lo = (float)(b[i] & 0x0F);
      float hi = (float)((b[i] >> 4) & 0x0F);
      out.push_back(lo * scale + zero);
      out.push_back(hi * scale + zero);
    }
  }
}

struct QuantCache {  // :14-36
  std::vector<std::vector<uint8_t>> keys, values;
  std::vector<std::vector<float>> kscale, vscale, kzero, vzero;
  size_t layers, heads, hd;
  int bits;
  size_t gs;
  size_t seq_len = 0;
  QuantCache(size_t l, size_t h, size_t d, int b, size_t g)
      : keys(l), values(l), kscale(l), vscale(l), kzero(l), vzero(l), layers(l), heads(h), hd(d), bits(b), gs(g) {}

  void quantize_data(const float* d, size_t n, std::vector<uint8_t>& bytes, std::vector<float>& sc,
                     std::vector<float>& zr) const {  // :177-197
    size_t ng = (n + gs - 1) / gs;
    for (size_t g = 0; g < ng; ++g) {
      size_t s = g * gs, e = s + gs < n ? s + gs : n;
      float a, z;
      quantize_group(d + s, e - s, bits, bytes, &a, &z);
      sc.push_back(a);
      zr.push_back(z);
    }
  }
  int append(size_t layer, const float* k, const float* v, size_t n_elems, size_t new_tokens) {  // :89-127
    if (layer >= layers) return ORC_E_RANGE;
    if (n_elems != heads * new_tokens * hd) return ORC_E_BAD_ARG;
    quantize_data(k, n_elems, keys[layer], kscale[layer], kzero[layer]);
    quantize_data(v, n_elems, values[layer], vscale[layer], vzero[layer]);
    if (layer == 0) seq_len += new_tokens;
    return ORC_OK;
  }
  // dequantize_data, :200-223.  Returns ORC_E_BAD_ARG where the Rust slice
  // indexing would panic (a group that starts past the end of the bytes).
  int dequantize(const std::vector<uint8_t>& b, const std::vector<float>& sc, const std::vector<float>& zr,
                 std::vector<float>& out) const {
    out.clear();
    if (b.empty()) return ORC_OK;
    size_t bpg = bits == 4 ? (gs + 1) / 2 : gs;
    for (size_t g = 0; g < sc.size(); ++g) {
      size_t s = g * bpg, e = s + bpg < b.size() ? s + bpg : b.size();
      if (s > e) return ORC_E_BAD_ARG;
      dequantize_group(b.data() + s, e - s, sc[g], zr[g], bits, out);
    }
    return ORC_OK;
  }
};

// ---------------------------------------------------------------------------
// RotatingKVCache -- rotating_cache.rs:16-283 (f32 storage)
// ---------------------------------------------------------------------------
struct Rotating {
  std::vector<std::vector<std::vector<float>>> keys, values;
  size_t layers, heads, hd, max_size, keep, offset = 0, written = 0;
  Rotating(size_t l, size_t h, size_t d, size_t m, size_t k)  // :45-84
      : keys(l, std::vector<std::vector<float>>(h, std::vector<float>(m * d, 0.0f))),
        values(l, std::vector<std::vector<float>>(h, std::vector<float>(m * d, 0.0f))),
        layers(l), heads(h), hd(d), max_size(m), keep(k) {}
  size_t seq_len() const { return written < max_size ? written : max_size; }  // :202-204
  int append(size_t layer, const float* k, const float* v, size_t n_elems, size_t nt) {  // :94-143
    if (n_elems != heads * nt * hd) return ORC_E_BAD_ARG;
    size_t rot = max_size - keep;
    for (size_t tok = 0; tok < nt; ++tok) {
      size_t wp = written < max_size ? written : keep + offset;
      for (size_t h = 0; h < heads; ++h) {
        size_t src = (h * nt + tok) * hd, dst = wp * hd;
        memcpy(&keys[layer][h][dst], k + src, hd * sizeof(float));
        memcpy(&values[layer][h][dst], v + src, hd * sizeof(float));
      }
      if (written >= max_size) offset = (offset + 1) % rot;
      written += 1;
    }
    return ORC_OK;
  }
  // get_logical_order, :162-197.  Writes heads * seq_len * hd floats.
  void logical(size_t layer, bool vals, float* out) const {
    const auto& st = vals ? values : keys;
    size_t L = seq_len();
    for (size_t h = 0; h < heads; ++h) {
      const float* buf = st[layer][h].data();
      float* o = out + h * L * hd;
      if (written <= max_size) {
        memcpy(o, buf, L * hd * sizeof(float));
      } else {
        memcpy(o, buf, keep * hd * sizeof(float));
        o += keep * hd;
        size_t rot = max_size - keep;
        for (size_t i = 0; i < rot; ++i) {
          size_t p = (offset + i) % rot;
          memcpy(o, buf + (keep + p) * hd, hd * sizeof(float));
          o += hd;
        }
      }
    }
  }
  int trim(size_t n) {  // :213-262
    size_t sl = seq_len();
    size_t trimmable = sl > keep ? sl - keep : 0;
    if (n > trimmable) return ORC_E_RANGE;
    if (written <= max_size) {
      for (auto* st : {&keys, &values})
        for (auto& lb : *st)
          for (auto& hb : lb) {
            size_t src = (keep + n) * hd, dst = keep * hd, rem = (written - keep - n) * hd;
            if (rem > 0) memmove(&hb[dst], &hb[src], rem * sizeof(float));
          }
      written -= n;
    } else {
      size_t rot = max_size - keep;
      offset = (offset + n) % rot;
      written -= n;
    }
    return ORC_OK;
  }
};

// ---------------------------------------------------------------------------
// XXH64 (published algorithm by Y. Collet), restated; used by the chain hash.
// ---------------------------------------------------------------------------
static const uint64_t P1 = 0x9E3779B185EBCA87ULL, P2 = 0xC2B2AE3D27D4EB4FULL, P3 = 0x165667B19E3779F9ULL,
                      P4 = 0x85EBCA77C2B2AE63ULL, P5 = 0x27D4EB2F165667C5ULL;
static inline uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
static inline uint64_t rd64(const uint8_t* p) {
  uint64_t v;
  memcpy(&v, p, 8);
  return v;
}
static inline uint32_t rd32(const uint8_t* p) {
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
}
static inline uint64_t xround(uint64_t acc, uint64_t lane) {
  acc += lane * P2;
  acc = rotl(acc, 31);
  return acc * P1;
}
static inline uint64_t xmerge(uint64_t acc, uint64_t v) {
  acc ^= xround(0, v);
  return acc * P1 + P4;
}
uint64_t xxh64(const uint8_t* p, size_t len, uint64_t seed) {
  const uint8_t* end = p + len;
  uint64_t h;
  if (len >= 32) {
    uint64_t v1 = seed + P1 + P2, v2 = seed + P2, v3 = seed, v4 = seed - P1;
    const uint8_t* lim = end - 32;
    do {
      v1 = xround(v1, rd64(p));
      v2 = xround(v2, rd64(p + 8));
      v3 = xround(v3, rd64(p + 16));
      v4 = xround(v4, rd64(p + 24));
      p += 32;
    } while (p <= lim);
    h = rotl(v1, 1) + rotl(v2, 7) + rotl(v3, 12) + rotl(v4, 18);
    h = xmerge(h, v1);
    h = xmerge(h, v2);
    h = xmerge(h, v3);
    h = xmerge(h, v4);
  } else {
    h = seed + P5;
  }
  h += (uint64_t)len;
  while (p + 8 <= end) {
    h ^= xround(0, rd64(p));
    h = rotl(h, 27) * P1 + P4;
    p += 8;
  }
  if (p + 4 <= end) {
    h ^= (uint64_t)rd32(p) * P1;
    h = rotl(h, 23) * P2 + P3;
    p += 4;
  }
  while (p < end) {
    h ^= (uint64_t)(*p) * P5;
    h = rotl(h, 11) * P1;
    p += 1;
  }
  h ^= h >> 33;
  h *= P2;
  h ^= h >> 29;
  h *= P3;
  h ^= h >> 32;
  return h;
}

// ---------------------------------------------------------------------------
// Paged pool geometry shared by the data ops below.  Block-major layout:
// pool[block][layer][kv][head][slot][row], one (block,layer,kv,head) "tile"
// of tile_bytes.  For plain pools a row is head_dim elements of elem_bytes;
// for quantised pools a tile is codes[slot][row_code_bytes] followed by
// meta[slot][groups][2] (scale, zero) in f32 or f16.
// ---------------------------------------------------------------------------
struct Geo {
  int64_t layers, heads, hd, bs, nblocks, elem, bits, gs, meta_bytes;
  int64_t row_bytes() const { return bits ? hd * bits / 8 : hd * elem; }
  int64_t meta_row_bytes() const { return bits ? (hd / gs) * 2 * meta_bytes : 0; }
  int64_t tile_bytes() const {
    int64_t t = bs * row_bytes() + bs * meta_row_bytes();
    return (t + 15) / 16 * 16;
  }
  int64_t tile_off(int64_t blk, int64_t l, int64_t kv, int64_t h) const {
    return (((blk * layers + l) * 2 + kv) * heads + h) * tile_bytes();
  }
};

static inline float half_bits_to_f32(uint16_t b) {
  _Float16 h;
  memcpy(&h, &b, 2);
  return (float)h;
}
static inline uint16_t f32_to_half_bits(float f) {
  _Float16 h = (_Float16)f;
  uint16_t b;
  memcpy(&b, &h, 2);
  return b;
}
static inline float bf16_bits_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t f32_to_bf16_bits(float f) {
  __bf16 h = (__bf16)f;
  uint16_t b;
  memcpy(&b, &h, 2);
  return b;
}
// dtype codes shared with the tests: 0 = f32, 1 = f16, 2 = bf16
static inline float load_elem(const uint8_t* p, int dt) {
  if (dt == 0) {
    float f;
    memcpy(&f, p, 4);
    return f;
  }
  uint16_t b;
  memcpy(&b, p, 2);
  return dt == 1 ? half_bits_to_f32(b) : bf16_bits_to_f32(b);
}
static inline void store_elem(uint8_t* p, int dt, float f) {
  if (dt == 0) {
    memcpy(p, &f, 4);
    return;
  }
  uint16_t b = dt == 1 ? f32_to_half_bits(f) : f32_to_bf16_bits(f);
  memcpy(p, &b, 2);
}

}  // namespace orc

using namespace orc;

extern "C" {

// ---- paged_cache.rs ------------------------------------------------------
void* orc_mgr_new(size_t bs, size_t n) { return new PagedManager(bs, n); }
void orc_mgr_delete(void* m) { delete (PagedManager*)m; }
int orc_mgr_allocate(void* m, size_t* out) { return ((PagedManager*)m)->allocate(out) ? 1 : 0; }
int orc_mgr_free(void* m, size_t id) { return ((PagedManager*)m)->free_block(id); }
int orc_mgr_ref_count(void* m, size_t id, size_t* out) { return ((PagedManager*)m)->ref_count(id, out); }
int orc_mgr_increment_ref(void* m, size_t id) { return ((PagedManager*)m)->increment_ref(id); }
int orc_mgr_copy_on_write(void* m, size_t id, size_t* out, int* copied) {
  return ((PagedManager*)m)->copy_on_write(id, out, copied);
}
size_t orc_mgr_num_free(void* m) { return ((PagedManager*)m)->free_blocks.size(); }
size_t orc_mgr_num_allocated(void* m) {
  auto* p = (PagedManager*)m;
  return p->num_blocks - p->free_blocks.size();
}
int orc_mgr_register_hash(void* m, size_t id, uint64_t h) { return ((PagedManager*)m)->register_hash(id, h); }
int orc_mgr_lookup_hash(void* m, uint64_t h, size_t* out) { return ((PagedManager*)m)->lookup_hash(h, out) ? 1 : 0; }
int orc_mgr_append_tokens(void* m, size_t id, const uint32_t* t, size_t n) {
  return ((PagedManager*)m)->append_tokens(id, t, n);
}
// get_block (:249-251): returns 0 when out of range; else fills the view.
int orc_mgr_get_block(void* m, size_t id, size_t* ref, int* has_hash, uint64_t* hash, size_t* num_filled,
                      uint32_t* tokens, size_t cap, size_t* ntok) {
  auto* p = (PagedManager*)m;
  if (id >= p->num_blocks) return 0;
  const Block& b = p->blocks[id];
  *ref = b.ref_count;
  *has_hash = b.has_hash;
  *hash = b.hash;
  *num_filled = b.num_filled;
  *ntok = b.tokens.size();
  for (size_t i = 0; i < b.tokens.size() && i < cap; ++i) tokens[i] = b.tokens[i];
  return 1;
}

// ---- prefix_cache.rs -----------------------------------------------------
void* orc_prefix_new(size_t maxb) { return new PrefixCache(maxb); }
void orc_prefix_delete(void* p) { delete (PrefixCache*)p; }
size_t orc_prefix_lookup(void* p, const uint32_t* t, size_t n, size_t* out, size_t cap) {
  auto ids = ((PrefixCache*)p)->lookup(t, n);
  for (size_t i = 0; i < ids.size() && i < cap; ++i) out[i] = ids[i];
  return ids.size();
}
void orc_prefix_insert(void* p, const uint32_t* t, size_t n, const size_t* ids, size_t nb) {
  ((PrefixCache*)p)->insert(t, n, ids, nb);
}
// insert, reporting per block whether its node had no block (attached[i] = 1)
// and the block it replaced (replaced[i], -1 for none)
void orc_prefix_insert_report(void* p, const uint32_t* t, size_t n, const size_t* ids, size_t nb, int32_t* attached,
                              int64_t* replaced) {
  std::vector<int> a;
  std::vector<long long> r;
  ((PrefixCache*)p)->insert_report(t, n, ids, nb, &a, &r);
  for (size_t i = 0; i < nb; ++i) {
    attached[i] = a[i];
    replaced[i] = r[i];
  }
}
int orc_prefix_evict_lru(void* p, size_t* out) { return ((PrefixCache*)p)->evict_lru(out) ? 1 : 0; }
double orc_prefix_hit_rate(void* p) { return ((PrefixCache*)p)->hit_rate(); }
size_t orc_prefix_num_blocks(void* p) { return ((PrefixCache*)p)->num_blocks; }
size_t orc_prefix_num_nodes(void* p) { return ((PrefixCache*)p)->nodes.size(); }

// ---- memory.rs -----------------------------------------------------------
void* orc_mem_new(size_t maxb, size_t limit_mb, size_t bpb) { return new MemPrefix(maxb, limit_mb, bpb); }
void orc_mem_delete(void* p) { delete (MemPrefix*)p; }
void orc_mem_insert(void* p, const uint32_t* t, size_t n, const size_t* ids, size_t nb) {
  ((MemPrefix*)p)->insert(t, n, ids, nb);
}
size_t orc_mem_lookup(void* p, const uint32_t* t, size_t n, size_t* out, size_t cap) {
  auto ids = ((MemPrefix*)p)->pc.lookup(t, n);
  for (size_t i = 0; i < ids.size() && i < cap; ++i) out[i] = ids[i];
  return ids.size();
}
int orc_mem_evict_lru(void* p, size_t* out) { return ((MemPrefix*)p)->evict_lru(out) ? 1 : 0; }
int orc_mem_should_evict(void* p) { return ((MemPrefix*)p)->should_evict() ? 1 : 0; }
size_t orc_mem_usage(void* p) { return ((MemPrefix*)p)->usage; }
size_t orc_mem_limit(void* p) { return ((MemPrefix*)p)->limit; }
size_t orc_mem_num_blocks(void* p) { return ((MemPrefix*)p)->pc.num_blocks; }
size_t orc_mem_evicted(void* p, size_t* out, size_t cap) {
  auto& v = ((MemPrefix*)p)->evicted_log;
  for (size_t i = 0; i < v.size() && i < cap; ++i) out[i] = v[i];
  return v.size();
}

// ---- quantized_cache.rs --------------------------------------------------
// quantize_group on one group; returns number of bytes written.
size_t orc_quantize_group(const float* d, size_t n, int bits, uint8_t* out, float* scale, float* zero) {
  std::vector<uint8_t> b;
  quantize_group(d, n, bits, b, scale, zero);
  memcpy(out, b.data(), b.size());
  return b.size();
}
size_t orc_dequantize_group(const uint8_t* b, size_t nb, float scale, float zero, int bits, float* out) {
  std::vector<float> v;
  dequantize_group(b, nb, scale, zero, bits, v);
  memcpy(out, v.data(), v.size() * sizeof(float));
  return v.size();
}
void* orc_qcache_new(size_t l, size_t h, size_t d, int bits, size_t gs) {
  if (bits != 4 && bits != 8) return nullptr;  // :57-60
  if (!(d % gs == 0 || gs > d)) return nullptr;  // :61-65
  return new QuantCache(l, h, d, bits, gs);
}
void orc_qcache_delete(void* q) { delete (QuantCache*)q; }
int orc_qcache_append(void* q, size_t layer, const float* k, const float* v, size_t n, size_t nt) {
  return ((QuantCache*)q)->append(layer, k, v, n, nt);
}
size_t orc_qcache_seq_len(void* q) { return ((QuantCache*)q)->seq_len; }
// which: 0 keys, 1 values.  *n_out = number of floats; returns status.
int orc_qcache_get_dequantized(void* q, size_t layer, int which, float* out, size_t cap, size_t* n_out) {
  auto* c = (QuantCache*)q;
  std::vector<float> v;
  int rc = which ? c->dequantize(c->values[layer], c->vscale[layer], c->vzero[layer], v)
                 : c->dequantize(c->keys[layer], c->kscale[layer], c->kzero[layer], v);
  *n_out = v.size();
  for (size_t i = 0; i < v.size() && i < cap; ++i) out[i] = v[i];
  return rc;
}
// raw stored state for bit-exact comparison: bytes, scales, zeros
size_t orc_qcache_raw(void* q, size_t layer, int which, uint8_t* bytes, size_t bcap, float* sc, float* zr,
                      size_t gcap, size_t* ngroups) {
  auto* c = (QuantCache*)q;
  auto& b = which ? c->values[layer] : c->keys[layer];
  auto& s = which ? c->vscale[layer] : c->kscale[layer];
  auto& z = which ? c->vzero[layer] : c->kzero[layer];
  for (size_t i = 0; i < b.size() && i < bcap; ++i) bytes[i] = b[i];
  for (size_t i = 0; i < s.size() && i < gcap; ++i) {
    sc[i] = s[i];
    zr[i] = z[i];
  }
  *ngroups = s.size();
  return b.size();
}

// ---- rotating_cache.rs ---------------------------------------------------
void* orc_rot_new(size_t l, size_t h, size_t d, size_t m, size_t k) {
  if (k >= m) return nullptr;  // :52-55
  return new Rotating(l, h, d, m, k);
}
void orc_rot_delete(void* r) { delete (Rotating*)r; }
int orc_rot_append(void* r, size_t layer, const float* k, const float* v, size_t n, size_t nt) {
  return ((Rotating*)r)->append(layer, k, v, n, nt);
}
size_t orc_rot_seq_len(void* r) { return ((Rotating*)r)->seq_len(); }
void orc_rot_get(void* r, size_t layer, int vals, float* out) { ((Rotating*)r)->logical(layer, vals != 0, out); }
int orc_rot_trim(void* r, size_t n) { return ((Rotating*)r)->trim(n); }

// ---- chain hash (build-defined; see file header) -------------------------
uint64_t orc_xxh64(const uint8_t* p, size_t len, uint64_t seed) { return xxh64(p, len, seed); }
// tokens of request r are tokens[cu_tokens[r] .. cu_tokens[r+1]); its blocks
// are written at out[cu_blocks[r] ..], cu_blocks[r+1]-cu_blocks[r] =
// ceil(n_r / block_size).  Block b hashes le64(parent) || le32(tok[b*bs ..]),
// parent of block 0 = root[r].
void orc_hash_chains(const uint32_t* tokens, const int64_t* cu_tokens, const uint64_t* root, int64_t nreq,
                     int64_t bs, const int64_t* cu_blocks, uint64_t* out) {
  std::vector<uint8_t> msg(8 + 4 * bs);
  for (int64_t r = 0; r < nreq; ++r) {
    uint64_t parent = root[r];
    int64_t n = cu_tokens[r + 1] - cu_tokens[r];
    const uint32_t* t = tokens + cu_tokens[r];
    int64_t nb = (n + bs - 1) / bs;
    for (int64_t b = 0; b < nb; ++b) {
      int64_t cnt = (b + 1) * bs <= n ? bs : n - b * bs;
      memcpy(msg.data(), &parent, 8);
      memcpy(msg.data() + 8, t + b * bs, 4 * cnt);
      parent = xxh64(msg.data(), 8 + 4 * cnt, 0);
      out[cu_blocks[r] + b] = parent;
    }
  }
}

// ---- paged K/V data ops (build-defined, rotating_cache.rs:126-136 row copy)
// geo: layers, heads, head_dim, block_size, num_blocks, elem_bytes, bits,
// group_size, meta_bytes (4 = f32, 2 = f16).
static Geo mkgeo(const int64_t* g) { return Geo{g[0], g[1], g[2], g[3], g[4], g[5], g[6], g[7], g[8]}; }

int64_t orc_tile_bytes(const int64_t* g) { return mkgeo(g).tile_bytes(); }

// Append n_tokens rows for layers [l0, l0+nl).  Source row (l, t, h) of k/v
// starts at byte ((l-l0)*ls + t*ts + h*hs) * elem.  slot < 0 skips the token.
// Returns 1 if a slot was out of range (that token is skipped), else 0.
int orc_paged_append(uint8_t* pool, const int64_t* g, int64_t l0, int64_t nl, const uint8_t* k, const uint8_t* v,
                     int64_t ls, int64_t ts, int64_t hs, const int64_t* slots, int64_t nt) {
  Geo G = mkgeo(g);
  int err = 0;
  int64_t rb = G.row_bytes();
  for (int64_t l = 0; l < nl; ++l)
    for (int64_t t = 0; t < nt; ++t) {
      int64_t s = slots[t];
      if (s < 0) continue;
      if (s >= G.nblocks * G.bs) {
        err = 1;
        continue;
      }
      int64_t blk = s / G.bs, off = s % G.bs;
      for (int kv = 0; kv < 2; ++kv)
        for (int64_t h = 0; h < G.heads; ++h) {
          const uint8_t* src = (kv ? v : k) + (l * ls + t * ts + h * hs) * G.elem;
          memcpy(pool + G.tile_off(blk, l0 + l, kv, h) + off * rb, src, rb);
        }
    }
  return err;
}

// Gather layer `layer` for `nseq` sequences into out_k/out_v laid out
// [seq][head][len][row], sequences packed back to back.  Returns 1 if a
// block-table entry was out of range (those rows are left untouched).
static int gather_range(const uint8_t* pool, const Geo& G, int64_t layer, const int32_t* bt, int64_t bt_stride,
                        const int32_t* lens, int64_t s0, int64_t s1, const int64_t* cu, uint8_t* ok, uint8_t* ov) {
  int err = 0;
  int64_t rb = G.row_bytes();
  for (int64_t s = s0; s < s1; ++s) {
    int64_t L = lens[s];
    for (int kv = 0; kv < 2; ++kv) {
      uint8_t* out = kv ? ov : ok;
      for (int64_t h = 0; h < G.heads; ++h) {
        uint8_t* o = out + (cu[s] * G.heads + h * L) * rb;
        for (int64_t t = 0; t < L; ++t) {
          int64_t blk = bt[s * bt_stride + t / G.bs];
          if (blk < 0 || blk >= G.nblocks) {
            err = 1;
            continue;
          }
          memcpy(o + t * rb, pool + G.tile_off(blk, layer, kv, h) + (t % G.bs) * rb, rb);
        }
      }
    }
  }
  return err;
}

int orc_paged_gather(const uint8_t* pool, const int64_t* g, int64_t layer, const int32_t* bt, int64_t bt_stride,
                     const int32_t* lens, int64_t nseq, uint8_t* ok, uint8_t* ov) {
  Geo G = mkgeo(g);
  std::vector<int64_t> cu(nseq + 1, 0);
  for (int64_t s = 0; s < nseq; ++s) cu[s + 1] = cu[s] + lens[s];
  return gather_range(pool, G, layer, bt, bt_stride, lens, 0, nseq, cu.data(), ok, ov);
}

// Same as orc_paged_gather, sequences split over `threads` host threads.
// Used only to time the CPU baseline on all host cores.
int orc_paged_gather_mt(const uint8_t* pool, const int64_t* g, int64_t layer, const int32_t* bt,
                        int64_t bt_stride, const int32_t* lens, int64_t nseq, uint8_t* ok, uint8_t* ov,
                        int threads) {
  Geo G = mkgeo(g);
  std::vector<int64_t> cu(nseq + 1, 0);
  for (int64_t s = 0; s < nseq; ++s) cu[s + 1] = cu[s] + lens[s];
  if (threads <= 1) return gather_range(pool, G, layer, bt, bt_stride, lens, 0, nseq, cu.data(), ok, ov);
  // balance by token count
  std::vector<int64_t> cuts(threads + 1, nseq);
  cuts[0] = 0;
  int64_t total = cu[nseq], ti = 1;
  for (int64_t s = 0; s < nseq && ti < threads; ++s)
    if (cu[s + 1] * threads >= total * ti) cuts[ti++] = s + 1;
  std::vector<int> errs(threads, 0);
  std::vector<std::thread> th;
  for (int i = 0; i < threads; ++i)
    th.emplace_back([&, i] {
      errs[i] = gather_range(pool, G, layer, bt, bt_stride, lens, cuts[i], cuts[i + 1], cu.data(), ok, ov);
    });
  for (auto& t : th) t.join();
  int e = 0;
  for (int x : errs) e |= x;
  return e;
}

// Block copy (copy-on-write data move): every tile of block src[i] -> dst[i].
int orc_copy_blocks(uint8_t* pool, const int64_t* g, const int32_t* src, const int32_t* dst, int64_t n) {
  Geo G = mkgeo(g);
  int64_t bb = G.tile_bytes() * G.layers * 2 * G.heads;
  int err = 0;
  for (int64_t i = 0; i < n; ++i) {
    if (src[i] < 0 || src[i] >= G.nblocks || dst[i] < 0 || dst[i] >= G.nblocks) {
      err = 1;
      continue;
    }
    memmove(pool + dst[i] * bb, pool + src[i] * bb, bb);
  }
  return err;
}

// Quantise-on-append into a quantised pool: each (layer, kv, token, head)
// row of head_dim elements (dtype in_dt) is converted to f32 and split into
// head_dim/gs groups, each quantised with quantize_group (:232-273).  Codes
// go to the tile's code row, (scale, zero) to its meta row in f32 or
// rounded to f16 (meta_bytes 2).
int orc_paged_append_quant(uint8_t* pool, const int64_t* g, int64_t l0, int64_t nl, const uint8_t* k,
                           const uint8_t* v, int in_dt, int64_t ls, int64_t ts, int64_t hs, const int64_t* slots,
                           int64_t nt) {
  Geo G = mkgeo(g);
  int64_t ies = in_dt == 0 ? 4 : 2;
  int64_t rb = G.row_bytes(), mrb = G.meta_row_bytes(), ng = G.hd / G.gs;
  std::vector<float> row(G.hd);
  int err = 0;
  for (int64_t l = 0; l < nl; ++l)
    for (int64_t t = 0; t < nt; ++t) {
      int64_t s = slots[t];
      if (s < 0) continue;
      if (s >= G.nblocks * G.bs) {
        err = 1;
        continue;
      }
      int64_t blk = s / G.bs, off = s % G.bs;
      for (int kv = 0; kv < 2; ++kv)
        for (int64_t h = 0; h < G.heads; ++h) {
          const uint8_t* src = (kv ? v : k) + (l * ls + t * ts + h * hs) * ies;
          for (int64_t d = 0; d < G.hd; ++d) row[d] = load_elem(src + d * ies, in_dt);
          uint8_t* tile = pool + G.tile_off(blk, l0 + l, kv, h);
          uint8_t* codes = tile + off * rb;
          uint8_t* meta = tile + G.bs * rb + off * mrb;
          std::vector<uint8_t> bytes;
          for (int64_t q = 0; q < ng; ++q) {
            float sc, zr;
            quantize_group(row.data() + q * G.gs, G.gs, (int)G.bits, bytes, &sc, &zr);
            if (G.meta_bytes == 4) {
              memcpy(meta + q * 8, &sc, 4);
              memcpy(meta + q * 8 + 4, &zr, 4);
            } else {
              uint16_t a = f32_to_half_bits(sc), b = f32_to_half_bits(zr);
              memcpy(meta + q * 4, &a, 2);
              memcpy(meta + q * 4 + 2, &b, 2);
            }
          }
          memcpy(codes, bytes.data(), rb);
        }
    }
  return err;
}

// Dequantise-on-gather: like orc_paged_gather, rows are dequantised with
// dequantize_group (:278-296) using the stored meta, then stored as out_dt.
static int gather_dq_range(const uint8_t* pool, const Geo& G, int64_t layer, const int32_t* bt,
                           int64_t bt_stride, const int32_t* lens, int64_t s0, int64_t s1, const int64_t* cu,
                           uint8_t* ok, uint8_t* ov, int out_dt) {
  int64_t oes = out_dt == 0 ? 4 : 2;
  int64_t rb = G.row_bytes(), mrb = G.meta_row_bytes(), ng = G.hd / G.gs;
  int64_t cpg = G.gs * G.bits / 8;  // code bytes per group
  std::vector<float> vals;
  int err = 0;
  for (int64_t s = s0; s < s1; ++s) {
    int64_t L = lens[s];
    for (int kv = 0; kv < 2; ++kv) {
      uint8_t* out = kv ? ov : ok;
      for (int64_t h = 0; h < G.heads; ++h) {
        uint8_t* o = out + (cu[s] * G.heads + h * L) * G.hd * oes;
        for (int64_t t = 0; t < L; ++t) {
          int64_t blk = bt[s * bt_stride + t / G.bs];
          if (blk < 0 || blk >= G.nblocks) {
            err = 1;
            continue;
          }
          const uint8_t* tile = pool + G.tile_off(blk, layer, kv, h);
          const uint8_t* codes = tile + (t % G.bs) * rb;
          const uint8_t* meta = tile + G.bs * rb + (t % G.bs) * mrb;
          vals.clear();
          for (int64_t q = 0; q < ng; ++q) {
            float sc, zr;
            if (G.meta_bytes == 4) {
              memcpy(&sc, meta + q * 8, 4);
              memcpy(&zr, meta + q * 8 + 4, 4);
            } else {
              uint16_t a, b;
              memcpy(&a, meta + q * 4, 2);
              memcpy(&b, meta + q * 4 + 2, 2);
              sc = half_bits_to_f32(a);
              zr = half_bits_to_f32(b);
            }
            dequantize_group(codes + q * cpg, cpg, sc, zr, (int)G.bits, vals);
          }
          for (int64_t d = 0; d < G.hd; ++d) store_elem(o + (t * G.hd + d) * oes, out_dt, vals[d]);
        }
      }
    }
  }
  return err;
}

int orc_paged_gather_dequant(const uint8_t* pool, const int64_t* g, int64_t layer, const int32_t* bt,
                             int64_t bt_stride, const int32_t* lens, int64_t nseq, uint8_t* ok, uint8_t* ov,
                             int out_dt, int threads) {
  Geo G = mkgeo(g);
  std::vector<int64_t> cu(nseq + 1, 0);
  for (int64_t s = 0; s < nseq; ++s) cu[s + 1] = cu[s] + lens[s];
  if (threads <= 1) return gather_dq_range(pool, G, layer, bt, bt_stride, lens, 0, nseq, cu.data(), ok, ov, out_dt);
  std::vector<int64_t> cuts(threads + 1, nseq);
  cuts[0] = 0;
  int64_t total = cu[nseq], ti = 1;
  for (int64_t s = 0; s < nseq && ti < threads; ++s)
    if (cu[s + 1] * threads >= total * ti) cuts[ti++] = s + 1;
  std::vector<int> errs(threads, 0);
  std::vector<std::thread> th;
  for (int i = 0; i < threads; ++i)
    th.emplace_back([&, i] {
      errs[i] = gather_dq_range(pool, G, layer, bt, bt_stride, lens, cuts[i], cuts[i + 1], cu.data(), ok, ov, out_dt);
    });
  for (auto& t : th) t.join();
  int e = 0;
  for (int x : errs) e |= x;
  return e;
}

// Prefix-cache admission driver (build-defined policy; the reference never
// connects PagedCacheManager and PrefixCacheManager).  Per request: LRU touch
// by prefix lookup of the full-block tokens; reuse of every full block whose
// chain hash is registered (request reference); allocation of the rest with
// LRU eviction from the prefix cache while the pool is empty (reject when
// nothing is left to evict); token ids and hashes of new blocks; insertion
// of the full-block prefix with one cache reference per newly held block;
// release of the request's references.  stats: requests, admitted, rejected,
// hit_blocks, new_blocks, evictions, lookup_tokens.
int orc_prefix_admit(void* mv, void* pv, const uint32_t* tokens, const int64_t* cu_tokens, const uint64_t* hashes,
                     const int64_t* cu_blocks, int64_t nreq, int64_t* block_ids, int64_t* evicted, int64_t cap,
                     int64_t* n_evicted, int64_t* stats) {
  auto* m = (PagedManager*)mv;
  auto* p = (PrefixCache*)pv;
  int64_t bs = (int64_t)m->block_size;
  for (int i = 0; i < 7; ++i) stats[i] = 0;
  *n_evicted = 0;
  std::vector<int> attached;
  std::vector<long long> replaced;
  for (int64_t r = 0; r < nreq; ++r) {
    int64_t n = cu_tokens[r + 1] - cu_tokens[r];
    const uint32_t* t = tokens + cu_tokens[r];
    const uint64_t* h = hashes + cu_blocks[r];
    int64_t* ids = block_ids + cu_blocks[r];
    int64_t nb = cu_blocks[r + 1] - cu_blocks[r];
    int64_t nfull = n / bs;
    stats[0] += 1;
    stats[6] += nfull * bs;
    p->lookup(t, (size_t)(nfull * bs));
    for (int64_t b = 0; b < nb; ++b) {
      ids[b] = -1;
      size_t id;
      if (b < nfull && m->lookup_hash(h[b], &id)) {
        m->increment_ref(id);
        ids[b] = (int64_t)id;
        stats[3] += 1;
      }
    }
    bool rejected = false;
    for (int64_t b = 0; b < nb && !rejected; ++b) {
      if (ids[b] >= 0) continue;
      size_t id;
      while (!m->allocate(&id)) {
        size_t victim;
        if (!p->evict_lru(&victim)) {
          rejected = true;
          break;
        }
        m->free_block(victim);
        if (*n_evicted < cap) evicted[*n_evicted] = (int64_t)victim;
        *n_evicted += 1;
        stats[5] += 1;
      }
      if (rejected) break;
      ids[b] = (int64_t)id;
      stats[4] += 1;
      int64_t cnt = (b + 1) * bs <= n ? bs : n - b * bs;
      m->append_tokens(id, t + b * bs, (size_t)cnt);
      if (b < nfull) m->register_hash(id, h[b]);
    }
    if (rejected) {
      for (int64_t b = 0; b < nb; ++b)
        if (ids[b] >= 0) m->free_block((size_t)ids[b]);
      for (int64_t b = 0; b < nb; ++b) ids[b] = -1;
      stats[2] += 1;
      continue;
    }
    if (nfull > 0) {
      std::vector<size_t> full(ids, ids + nfull);
      p->insert_report(t, (size_t)(nfull * bs), full.data(), (size_t)nfull, &attached, &replaced);
      for (int64_t b = 0; b < nfull; ++b) {
        // the cache holds one reference on every block it holds: a block it
        // starts holding (new node block, or one that replaces another) gains
        // one, a block it stops holding loses one
        if (attached[b] || replaced[b] >= 0) m->increment_ref((size_t)ids[b]);
        if (replaced[b] >= 0) m->free_block((size_t)replaced[b]);
      }
    }
    for (int64_t b = 0; b < nb; ++b) m->free_block((size_t)ids[b]);
    stats[1] += 1;
  }
  return ORC_OK;
}

// Element conversions used by tests (RNE, same as the reference's f32 path
// followed by a storage rounding).
void orc_f32_to_dtype(const float* in, uint8_t* out, int64_t n, int dt) {
  int64_t es = dt == 0 ? 4 : 2;
  for (int64_t i = 0; i < n; ++i) store_elem(out + i * es, dt, in[i]);
}
void orc_dtype_to_f32(const uint8_t* in, float* out, int64_t n, int dt) {
  int64_t es = dt == 0 ? 4 : 2;
  for (int64_t i = 0; i < n; ++i) out[i] = load_elem(in + i * es, dt);
}

}  // extern "C"
