// Host-side layout builders of the chain-of-edits attention (C ABI in
// include/ai_attn.h; no GPU involved).
//
// ai_attn_positions_from_ops: an edit chain -> the concat()-ed arrays of its
//   position-block list.  Restates, in one pass over plain arrays, the
//   reference's perturb_labels_per_sequence (perturb_labels.py:236-275: the
//   token index bookkeeping of each operation) and
//   get_parsed_positions_from_perturbations (perturb_labels.py:395-467: the
//   running position ids, abs mask and attention mask, and the EXTEND / EDIT /
//   COMPLETE blocks pushed from them), followed by PositionBlockList.concat()
//   (perturb_labels.py:341-357).  The reference runs these as per-operation
//   torch ops on the training device with a host sync per operation.
//
// ai_attn_prep: concat()-ed lists (one per batch row, or shared) -> the
//   device tables of AiAttnLayout (block records, key words, query / own-key
//   table rows, forward and dK/dV work lists, counts), written into host
//   buffers the caller copies to the device in one transfer.

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <unordered_map>
#include <vector>

#include "../../include/ai_attn.h"

namespace {

struct Op {
  int64_t num_insert, num_delete, start_rel_pos, end_rel_pos, num_extend;
};

// One pushed block: [start, end) query rows; key arrays are the snapshots of
// the running arrays over [0, end) at push time.
struct PushedBlock {
  int64_t start, end;
  int32_t type;  // AI_BLOCK_TYPE_*
  std::vector<int64_t> key_pos;
  std::vector<uint8_t> attn, abs;
  std::vector<int64_t> query_pos;
};

// Replays the operations; fills `blocks` (when not null) and returns
// AI_OK, or AI_ERR_LAYOUT for an operation list the reference rejects.
int replay_ops(const Op* ops, int n_ops, std::vector<PushedBlock>* blocks, int64_t* token_count_out,
               int32_t* n_blocks_out, int64_t* n_keys_out) {
  if (n_ops <= 0) return AI_ERR_LAYOUT;
  // perturb_labels_per_sequence: lengths and marker indices per operation.
  struct Pert {
    int64_t edit_idx, return_idx, post_len;
    bool edit;
  };
  std::vector<Pert> perts((size_t)n_ops);
  int64_t len = 0, cur = 0;  // len(token_indices), curr_seq_idx
  for (int i = 0; i < n_ops; ++i) {
    const Op& op = ops[i];
    if (op.num_insert < 0 || op.num_delete < 0 || op.num_extend < 0) return AI_ERR_LAYOUT;
    Pert p{-1, -1, 0, false};
    if (op.num_insert > 0 || op.num_delete > 0) {
      // an edit needs a token before it and a valid cursor range
      if (cur <= 0 || op.start_rel_pos < 0 || op.start_rel_pos > op.end_rel_pos || op.start_rel_pos >= len ||
          op.end_rel_pos > len)
        return AI_ERR_LAYOUT;
      p.edit = true;
      p.edit_idx = cur;
      p.return_idx = cur + op.num_insert + 1;
      len = len - (op.end_rel_pos - op.start_rel_pos) + op.num_insert;
      cur += op.num_insert + 2;
    }
    p.post_len = len;
    len += op.num_extend;
    cur += op.num_extend;
    perts[(size_t)i] = p;
  }
  const int64_t T = cur;  // token_count
  if (T <= 0 || T > (int64_t)1 << 30) return AI_ERR_LAYOUT;
  std::vector<int64_t> pos((size_t)T, 0);
  std::vector<uint8_t> absm((size_t)T, 0), attn((size_t)T, 1);
  int64_t start = 0, n_keys = 0;
  int32_t n_blocks = 0;
  auto push = [&](int64_t end, int32_t type) -> int {
    if (end <= start || end > T) return AI_ERR_LAYOUT;
    if (type == AI_BLOCK_TYPE_EXTEND) {
      int64_t attended = 0;
      for (int64_t j = 0; j < end; ++j) attended += attn[(size_t)j];
      if (attended <= 1 || end < 2) return AI_ERR_LAYOUT;  // an edit marker cannot open the sequence
    }
    if (blocks) {
      PushedBlock b;
      b.start = start;
      b.end = end;
      b.type = type;
      b.key_pos.assign(pos.begin(), pos.begin() + end);
      if (type == AI_BLOCK_TYPE_EXTEND) b.key_pos[(size_t)end - 1] = b.key_pos[(size_t)end - 2] + 1;
      b.attn.assign(attn.begin(), attn.begin() + end);
      for (int64_t j = 0; j < end; ++j)
        if (!b.attn[(size_t)j]) b.key_pos[(size_t)j] = -1;
      if (type == AI_BLOCK_TYPE_EDIT)
        b.abs.assign(absm.begin(), absm.begin() + end);
      else
        b.abs.assign((size_t)end, 0);
      b.query_pos.assign(pos.begin() + start, pos.begin() + end);
      blocks->push_back(std::move(b));
    }
    n_keys += end;
    ++n_blocks;
    start = end;
    return AI_OK;
  };
  for (int i = 0; i < n_ops; ++i) {
    const Op& op = ops[i];
    const Pert& pt = perts[(size_t)i];
    if (pt.edit) {
      const int64_t ed = pt.edit_idx, rt = pt.return_idx;
      if (rt >= T) return AI_ERR_LAYOUT;
      pos[(size_t)ed] = op.start_rel_pos - 1;
      for (int64_t j = 0; j < ed; ++j) absm[(size_t)j] = pos[(size_t)j] >= op.start_rel_pos;
      absm[(size_t)ed] = 1;
      for (int64_t j = 0; j < T; ++j) absm[(size_t)j] &= attn[(size_t)j];
      int rc = push(ed + 1, AI_BLOCK_TYPE_EXTEND);
      if (rc != AI_OK) return rc;
      for (int64_t j = 0; j < T; ++j)
        if (absm[(size_t)j]) pos[(size_t)j] += 1 - op.start_rel_pos;
      for (int64_t j = 0; j < T; ++j)
        if (absm[(size_t)j] && pos[(size_t)j] > op.num_delete) pos[(size_t)j] += 1;
      pos[(size_t)ed] = op.num_delete + 1;
      if (op.num_insert > 0) {
        for (int64_t j = start; j < rt; ++j) pos[(size_t)j] = op.start_rel_pos + (j - start);
        rc = push(rt, AI_BLOCK_TYPE_EDIT);
        if (rc != AI_OK) return rc;
      }
      for (int64_t j = 0; j < T; ++j)
        if (absm[(size_t)j]) pos[(size_t)j] += op.start_rel_pos + op.num_insert - op.num_delete - 2;
      pos[(size_t)rt] = pt.post_len - 1;
      const int64_t pe = pos[(size_t)ed];
      for (int64_t j = 0; j < T; ++j)
        if (absm[(size_t)j] && pos[(size_t)j] <= pe) attn[(size_t)j] = 0;
      attn[(size_t)rt] = 0;
      std::fill(absm.begin(), absm.end(), 0);
    }
    const int64_t ext_pos = start > 0 ? pos[(size_t)start] + 1 : 0;
    const int64_t ext_idx = start > 0 ? start + 1 : 0;
    for (int64_t x = 0; x < op.num_extend && ext_idx + x < T; ++x) pos[(size_t)(ext_idx + x)] = ext_pos + x;
  }
  int rc = push(T, AI_BLOCK_TYPE_COMPLETE);
  if (rc != AI_OK) return rc;
  *token_count_out = T;
  *n_blocks_out = n_blocks;
  *n_keys_out = n_keys;
  return AI_OK;
}

// ------------------------------------------------------------------ ai_attn_prep

struct ListView {
  const AiPrepList* l;
  std::vector<uint32_t> info;   // key words (table row | attn | abs)
  std::vector<int32_t> own;     // [seq_len] own-block table row of each key
  std::vector<uint8_t> own_ok;  // per block: every attended key at its own-block row
  int64_t pairs = 0;
  int64_t key_base = 0;
};

int check_list(const AiPrepList& l, int32_t seq_len) {
  if (l.n_blocks <= 0 || !l.boundary || !l.query_pos || !l.key_pos || !l.attn_mask) return AI_ERR_NULL;
  int64_t expect = 0;
  for (int32_t i = 0; i < l.n_blocks; ++i) {
    const int64_t* b = l.boundary + 4 * (int64_t)i;
    if (b[0] != expect || b[1] <= b[0] || b[3] - b[2] != b[1] || b[1] > seq_len) return AI_ERR_LAYOUT;
    if (i > 0 && b[2] != l.boundary[4 * (int64_t)(i - 1) + 3]) return AI_ERR_LAYOUT;
    if (i == 0 && b[2] != 0) return AI_ERR_LAYOUT;
    expect = b[1];
  }
  if (l.n_query != expect) return AI_ERR_LAYOUT;
  if (l.n_keys != l.boundary[4 * (int64_t)(l.n_blocks - 1) + 3]) return AI_ERR_LAYOUT;
  return AI_OK;
}

struct Plan {
  int64_t lo = 0, hi = 0, n_keys = 0;
  int32_t n_blocks = 0, n_fwd = 0, n_kv = 0;
};

int plan(const AiPrepList* lists, int32_t n_lists, const int32_t* list_of_row, int32_t batch, int32_t seq_len,
         int32_t fwd_tile, int32_t kv_tile, Plan* p) {
  if (!lists || !list_of_row || !p) return AI_ERR_NULL;
  if (n_lists <= 0 || batch <= 0 || seq_len <= 0 || fwd_tile <= 0 || kv_tile <= 0) return AI_ERR_SHAPE;
  for (int32_t u = 0; u < n_lists; ++u) {
    int rc = check_list(lists[u], seq_len);
    if (rc != AI_OK) return rc;
  }
  Plan q;
  for (int32_t u = 0; u < n_lists; ++u) {
    const AiPrepList& l = lists[u];
    for (int64_t i = 0; i < l.n_query; ++i) {
      q.lo = std::min(q.lo, l.query_pos[i]);
      q.hi = std::max(q.hi, l.query_pos[i]);
    }
    for (int64_t j = 0; j < l.n_keys; ++j)
      if (l.attn_mask[j]) {
        q.lo = std::min(q.lo, l.key_pos[j]);
        q.hi = std::max(q.hi, l.key_pos[j]);
      }
    q.n_keys += l.n_keys;
  }
  if (q.hi - q.lo + 1 > (int64_t)AI_KEY_ROW_MASK) return AI_ERR_LAYOUT;
  for (int32_t b = 0; b < batch; ++b) {
    const int32_t u = list_of_row[b];
    if (u < 0 || u >= n_lists) return AI_ERR_LAYOUT;
    const AiPrepList& l = lists[u];
    q.n_blocks += l.n_blocks;
    for (int32_t i = 0; i < l.n_blocks; ++i) {
      const int64_t s = l.boundary[4 * (int64_t)i], e = l.boundary[4 * (int64_t)i + 1];
      q.n_fwd += (int32_t)((e - s + fwd_tile - 1) / fwd_tile);
    }
    q.n_kv += (int32_t)((l.n_query + kv_tile - 1) / kv_tile);
  }
  *p = q;
  return AI_OK;
}

// Every table of a layout, in host vectors.
struct Tables {
  std::vector<int32_t> blocks, row_blocks, row_cov, q_pos, k_own, fwd_items, kv_items, kv_chunks, kv_reduce;
  std::vector<int32_t> blk_cls, chunk_cls, rot_classes;
  std::vector<uint32_t> key_info;
  int32_t n_fwd_abs = 0, n_fwd_abs_short = 0, n_fwd_short = 0, n_kv_abs = 0, n_kv_partials = 0, kv_cost_max = 0, kv_cost_total = 0;
  bool all_owned = true;
  int64_t pairs = 0, p_min = 0, p_max = 0;
};

// Query rows per step of the tensor-core dK/dV kernel, and its chunking costs.
constexpr int64_t kKvStepRows = 64, kSplitCost = 64, kChunkCost = 40;
// Keys per rotation-class chunk, and the most classes one layout gets
// (8192 classes x 8 KV heads x 16 KB = 1 GiB of rotated chunks); blocks
// past the cap rotate their keys in shared memory.
constexpr int64_t kClsKeys = 64;
constexpr int32_t kMaxRotClasses = 8192;

// Rotation classes: every 64-key chunk of a block without own positions
// (and with kv_lo on a chunk boundary) is described by its batch row, first
// key and, per key, the rotary table row (attended), kUnattended or kPast
// (at or past the block's end); equal descriptions share a class.
constexpr uint32_t kUnattended = 0xFFFFFFFEu, kPast = 0xFFFFFFFFu;

// FNV-1a over a chunk description's words.
inline uint64_t hash_words(const uint32_t* w, int n) {
  uint64_t h = 1469598103934665603ull;
  for (int i = 0; i < n; ++i) {
    h ^= w[i];
    h *= 1099511628211ull;
  }
  return h;
}

void build_rot_classes(Tables* t) {
  constexpr int kWords = 2 + (int)kClsKeys;  // batch row, first key, one word per key
  const int32_t nb = (int32_t)(t->blocks.size() / AI_BLOCK_FIELDS);
  t->blk_cls.assign((size_t)nb, -1);
  t->chunk_cls.clear();
  t->rot_classes.clear();
  std::vector<uint32_t> descs;                      // [class][kWords]
  std::unordered_multimap<uint64_t, int32_t> by_hash;
  std::vector<uint32_t> cur;                        // this block's chunk descriptions
  std::vector<int32_t> found;
  auto lookup = [&](const uint32_t* w, uint64_t h) -> int32_t {
    auto range = by_hash.equal_range(h);
    for (auto it = range.first; it != range.second; ++it)
      if (std::memcmp(descs.data() + (size_t)it->second * kWords, w, sizeof(uint32_t) * kWords) == 0)
        return it->second;
    return -1;
  };
  for (int32_t bi = 0; bi < nb; ++bi) {
    const int32_t* rec = t->blocks.data() + (int64_t)AI_BLOCK_FIELDS * bi;
    const int64_t e = rec[AI_BLOCK_END], kv_lo = rec[AI_BLOCK_KV_LO], off = rec[AI_BLOCK_KEY_OFF];
    if ((rec[AI_BLOCK_FLAGS] & AI_BLOCKF_OWNPOS) || kv_lo >= e || kv_lo % kClsKeys) continue;
    const int64_t n_chunks = 2 * ((e - kv_lo + 2 * kClsKeys - 1) / (2 * kClsKeys));
    const int64_t n_real = (e - kv_lo + kClsKeys - 1) / kClsKeys;
    cur.assign((size_t)(n_real * kWords), 0);
    found.assign((size_t)n_real, -1);
    std::vector<uint64_t> hashes((size_t)n_real);
    int32_t fresh = 0;
    for (int64_t i = 0; i < n_real; ++i) {
      const int64_t k0 = kv_lo + kClsKeys * i;
      uint32_t* w = cur.data() + (size_t)(i * kWords);
      w[0] = (uint32_t)rec[AI_BLOCK_ROW];
      w[1] = (uint32_t)k0;
      for (int64_t j = k0; j < k0 + kClsKeys; ++j) {
        uint32_t x = kPast;
        if (j < e) {
          const uint32_t kw = t->key_info[(size_t)(off + j)];
          x = (kw & AI_KEY_ATTN) ? (kw & AI_KEY_ROW_MASK) : kUnattended;
        }
        w[2 + (j - k0)] = x;
      }
      hashes[(size_t)i] = hash_words(w, kWords);
      found[(size_t)i] = lookup(w, hashes[(size_t)i]);
      fresh += found[(size_t)i] < 0;  // a block's own chunks differ in their first key
    }
    if ((int64_t)(descs.size() / kWords) + fresh > kMaxRotClasses) continue;
    t->blk_cls[(size_t)bi] = (int32_t)t->chunk_cls.size();
    int32_t last = -1;
    for (int64_t i = 0; i < n_real; ++i) {
      int32_t id = found[(size_t)i];
      if (id < 0) {
        id = (int32_t)(descs.size() / kWords);
        descs.insert(descs.end(), cur.begin() + i * kWords, cur.begin() + (i + 1) * kWords);
        by_hash.emplace(hashes[(size_t)i], id);
        t->rot_classes.push_back(bi);
        t->rot_classes.push_back((int32_t)(kv_lo + kClsKeys * i));
      }
      last = id;
      t->chunk_cls.push_back(id);
    }
    for (int64_t i = n_real; i < n_chunks; ++i) t->chunk_cls.push_back(last);  // padding of the last 128-key tile
  }
}

int build(const AiPrepList* lists, int32_t n_lists, const int32_t* list_of_row, int32_t batch, int32_t seq_len,
          int32_t fwd_tile, int32_t kv_tile, Tables* t) {
  Plan p;
  int rc = plan(lists, n_lists, list_of_row, batch, seq_len, fwd_tile, kv_tile, &p);
  if (rc != AI_OK) return rc;
  const int64_t lo = p.lo, n_pos = p.hi - p.lo + 1;
  auto row_of = [&](int64_t pos) -> uint32_t {
    int64_t r = pos - lo;
    r = r < 0 ? 0 : (r >= n_pos ? n_pos - 1 : r);
    return (uint32_t)r;
  };

  t->key_info.assign((size_t)p.n_keys, 0);
  // Per list: key words, own-block rows, OWNPOS per block, finite pairs.
  std::vector<ListView> views((size_t)n_lists);
  int64_t base = 0;
  for (int32_t u = 0; u < n_lists; ++u) {
    const AiPrepList& l = lists[u];
    ListView& v = views[(size_t)u];
    v.l = &l;
    v.key_base = base;
    base += l.n_keys;
    v.info.resize((size_t)l.n_keys);
    for (int64_t j = 0; j < l.n_keys; ++j) {
      const bool at = l.attn_mask[j] != 0, ab = l.abs_mask && l.abs_mask[j] && at;
      v.info[(size_t)j] = row_of(l.key_pos[j]) | (at ? AI_KEY_ATTN : 0u) | (ab ? AI_KEY_ABS : 0u);
    }
    v.own.assign((size_t)seq_len, 0);
    for (int32_t i = 0; i < l.n_blocks; ++i) {
      const int64_t* bd = l.boundary + 4 * (int64_t)i;
      for (int64_t r = bd[0]; r < bd[1]; ++r) v.own[(size_t)r] = (int32_t)(v.info[(size_t)(bd[2] + r)] & AI_KEY_ROW_MASK);
    }
    v.own_ok.resize((size_t)l.n_blocks);
    for (int32_t i = 0; i < l.n_blocks; ++i) {
      const int64_t* bd = l.boundary + 4 * (int64_t)i;
      bool ok = true;
      int64_t cum = 0;
      for (int64_t j = 0; j < bd[1]; ++j) {
        const uint32_t w = v.info[(size_t)(bd[2] + j)];
        if (w & AI_KEY_ATTN) {
          ++cum;
          if ((int32_t)(w & AI_KEY_ROW_MASK) != v.own[(size_t)j]) ok = false;
        }
        if (j >= bd[0]) v.pairs += cum;  // row j sees the attended keys up to j
      }
      v.own_ok[(size_t)i] = ok;
    }
    std::memcpy(t->key_info.data() + v.key_base, v.info.data(), sizeof(uint32_t) * (size_t)l.n_keys);
  }

  // Blocks, row tables, query / own rows.
  struct FwdItem {
    int64_t cost;
    int32_t block, q0, q1, group;
  };
  struct KvItem {
    int64_t cost;
    int32_t row, j0, j1;
    bool abs;
  };
  std::vector<FwdItem> fwd;
  std::vector<KvItem> kv;
  fwd.reserve((size_t)p.n_fwd);
  kv.reserve((size_t)p.n_kv);
  int32_t nb = 0;
  int64_t pairs = 0;
  bool all_owned = true;
  t->row_blocks.assign((size_t)batch + 1, 0);
  t->row_cov.assign((size_t)batch, 0);
  t->q_pos.assign((size_t)batch * seq_len, 0);
  t->k_own.assign((size_t)batch * seq_len, 0);
  t->blocks.assign((size_t)AI_BLOCK_FIELDS * p.n_blocks, 0);
  for (int32_t b = 0; b < batch; ++b) {
    const ListView& v = views[(size_t)list_of_row[b]];
    const AiPrepList& l = *v.l;
    const int32_t first = nb;
    for (int32_t i = 0; i < l.n_blocks; ++i) {
      const int64_t* bd = l.boundary + 4 * (int64_t)i;
      const int64_t s = bd[0], e = bd[1], ks = bd[2];
      int64_t kv_lo = e, abs_lo = 0, abs_hi = 0, last_att = -1;
      bool any_abs = false;
      for (int64_t j = 0; j < e; ++j) {
        const uint32_t w = v.info[(size_t)(ks + j)];
        if (w & AI_KEY_ATTN) {
          if (kv_lo == e) kv_lo = j;
          last_att = j;
        }
        if (w & AI_KEY_ABS) {
          if (!any_abs) abs_lo = j;
          abs_hi = j + 1;
          any_abs = true;
        }
      }
      int32_t flags = 0;
      if (kv_lo < e) {
        int64_t attended = 0;
        for (int64_t j = kv_lo; j < e; ++j) attended += (v.info[(size_t)(ks + j)] & AI_KEY_ATTN) ? 1 : 0;
        if (attended != e - kv_lo) flags |= AI_BLOCKF_MASKED;
      }
      (void)last_att;
      if (any_abs) flags |= AI_BLOCKF_ABS;
      if (v.own_ok[(size_t)i]) flags |= AI_BLOCKF_OWNPOS;
      int32_t* rec = t->blocks.data() + (int64_t)AI_BLOCK_FIELDS * nb;
      rec[AI_BLOCK_ROW] = b;
      rec[AI_BLOCK_START] = (int32_t)s;
      rec[AI_BLOCK_END] = (int32_t)e;
      rec[AI_BLOCK_KEY_OFF] = (int32_t)(v.key_base + ks);
      rec[AI_BLOCK_KV_LO] = (int32_t)kv_lo;
      rec[AI_BLOCK_FLAGS] = flags;
      rec[AI_BLOCK_ABS_LO] = (int32_t)abs_lo;
      rec[AI_BLOCK_ABS_HI] = (int32_t)abs_hi;
      for (int64_t q0 = s; q0 < e; q0 += fwd_tile) {
        const int64_t q1 = std::min<int64_t>(q0 + fwd_tile, e);
        const int64_t cost = (q1 - q0) * std::max<int64_t>(0, std::min(e, q1) - kv_lo);
        const bool short_item = q1 - q0 <= fwd_tile / 2;
        const int32_t group = (flags & AI_BLOCKF_ABS) ? (short_item ? 0 : 1) : (short_item ? 2 : 3);
        fwd.push_back({cost, nb, (int32_t)q0, (int32_t)q1, group});
      }
      ++nb;
    }
    t->row_blocks[(size_t)b + 1] = nb;
    const int64_t cov = l.n_query;
    t->row_cov[(size_t)b] = (int32_t)cov;
    if (cov < seq_len) all_owned = false;
    int32_t* qp = t->q_pos.data() + (int64_t)b * seq_len;
    int32_t* ko = t->k_own.data() + (int64_t)b * seq_len;
    const uint32_t zero_row = row_of(0);
    for (int64_t r = 0; r < seq_len; ++r) {
      qp[r] = (int32_t)(r < cov ? row_of(l.query_pos[r]) : zero_row);
      ko[r] = v.own[(size_t)r];
    }
    pairs += v.pairs;
    // Key tiles of this row: cost = query rows that see them; whether they
    // hold an abs key of some block.
    for (int64_t j0 = 0; j0 < cov; j0 += kv_tile) {
      const int64_t j1 = std::min<int64_t>(j0 + kv_tile, cov);
      int64_t cost = 0;
      bool abs = false;
      for (int32_t bi = first; bi < nb; ++bi) {
        const int32_t* rec = t->blocks.data() + (int64_t)AI_BLOCK_FIELDS * bi;
        const int64_t s = rec[AI_BLOCK_START], e = rec[AI_BLOCK_END];
        if (!(e > j0 && rec[AI_BLOCK_KV_LO] < j1)) continue;
        cost += std::max<int64_t>(e - std::max<int64_t>(s, j0), 0);
        if ((rec[AI_BLOCK_FLAGS] & AI_BLOCKF_ABS) && rec[AI_BLOCK_ABS_LO] < j1 && rec[AI_BLOCK_ABS_HI] > j0) abs = true;
      }
      kv.push_back({cost, b, (int32_t)j0, (int32_t)j1, abs});
    }
  }

  // Forward items: abs blocks' short items (at most fwd_tile / 2 rows), their
  // other items, then the other blocks' short items, then the rest; longest
  // first in each group (stable, so ties keep block order).
  std::stable_sort(fwd.begin(), fwd.end(), [](const FwdItem& x, const FwdItem& y) {
    if (x.group != y.group) return x.group < y.group;
    return x.cost > y.cost;
  });
  t->fwd_items.resize(4 * fwd.size());
  for (size_t i = 0; i < fwd.size(); ++i) {
    t->fwd_items[4 * i] = fwd[i].block;
    t->fwd_items[4 * i + 1] = fwd[i].q0;
    t->fwd_items[4 * i + 2] = fwd[i].q1;
    t->fwd_items[4 * i + 3] = 0;
    t->n_fwd_abs += fwd[i].group <= 1;
    t->n_fwd_abs_short += fwd[i].group == 0;
    t->n_fwd_short += fwd[i].group == 2;
  }
  std::stable_sort(kv.begin(), kv.end(), [](const KvItem& x, const KvItem& y) {
    if (x.abs != y.abs) return x.abs;
    return x.cost > y.cost;
  });
  t->kv_items.resize(4 * kv.size());
  for (size_t i = 0; i < kv.size(); ++i) {
    t->kv_items[4 * i] = kv[i].row;
    t->kv_items[4 * i + 1] = kv[i].j0;
    t->kv_items[4 * i + 2] = kv[i].j1;
    t->kv_items[4 * i + 3] = 0;
    t->n_kv_abs += kv[i].abs;
  }
  t->all_owned = all_owned;
  t->pairs = pairs;
  t->p_min = p.lo;
  t->p_max = p.hi;

  // dK/dV chunks: each key tile's 64-row query tiles (blocks without an abs
  // key among the tile's keys, block order), cost 1 a query tile and 2 a
  // block start; a tile costing more than kSplitCost is cut into chunks of
  // about kChunkCost (a chunk that starts inside a block pays its start).
  struct Chunk {
    int64_t cost;
    int32_t item, q0, q1, slot;
  };
  std::vector<Chunk> chunks;
  const bool any_abs_item = t->n_kv_abs > 0;
  for (size_t k = 0; k < kv.size(); ++k) {
    const int32_t b = kv[k].row, j0 = kv[k].j0, j1 = kv[k].j1;
    std::vector<int64_t> tile_cost;  // cost charged to each query tile, in order
    for (int32_t bi = t->row_blocks[(size_t)b]; bi < t->row_blocks[(size_t)b + 1]; ++bi) {
      const int32_t* rec = t->blocks.data() + (int64_t)AI_BLOCK_FIELDS * bi;
      const int64_t s = rec[AI_BLOCK_START], e = rec[AI_BLOCK_END];
      if (!(e > j0 && rec[AI_BLOCK_KV_LO] < j1 && std::max<int64_t>(s, j0) < e)) continue;
      if (any_abs_item && (rec[AI_BLOCK_FLAGS] & AI_BLOCKF_ABS)) {
        const int32_t lo = rec[AI_BLOCK_ABS_LO], hi = rec[AI_BLOCK_ABS_HI];
        if (hi <= lo || (j0 < hi && lo < j1)) continue;
      }
      const int64_t nq = (e - std::max<int64_t>(s, j0) + kKvStepRows - 1) / kKvStepRows;
      for (int64_t x = 0; x < nq; ++x) tile_cost.push_back(x == 0 ? 3 : 1);
    }
    int64_t total = 0;
    for (int64_t c : tile_cost) total += c;
    t->kv_cost_max = std::max<int32_t>(t->kv_cost_max, (int32_t)std::min<int64_t>(total, INT32_MAX));
    t->kv_cost_total = (int32_t)std::min<int64_t>((int64_t)t->kv_cost_total + total, INT32_MAX);
    const int32_t nqt = (int32_t)tile_cost.size();
    if (total <= kSplitCost) {
      chunks.push_back({total, (int32_t)k, 0, nqt, -1});
      continue;
    }
    int32_t first = (int32_t)chunks.size(), start = 0;
    int64_t acc = 0;
    for (int32_t x = 0; x < nqt; ++x) {
      acc += (x == start && tile_cost[(size_t)x] == 1) ? 3 : tile_cost[(size_t)x];
      if (acc >= kChunkCost && x + 1 < nqt) {
        chunks.push_back({acc, (int32_t)k, start, x + 1, 0});
        start = x + 1;
        acc = 0;
      }
    }
    chunks.push_back({acc, (int32_t)k, start, nqt, 0});
    const int32_t n = (int32_t)chunks.size() - first;
    for (int32_t c = 0; c < n; ++c) chunks[(size_t)(first + c)].slot = t->n_kv_partials + c;
    t->kv_reduce.insert(t->kv_reduce.end(), {(int32_t)k, t->n_kv_partials, n, 0});
    t->n_kv_partials += n;
  }
  std::stable_sort(chunks.begin(), chunks.end(), [](const Chunk& x, const Chunk& y) { return x.cost > y.cost; });
  t->kv_chunks.resize(4 * chunks.size());
  for (size_t i = 0; i < chunks.size(); ++i) {
    t->kv_chunks[4 * i] = chunks[i].item;
    t->kv_chunks[4 * i + 1] = chunks[i].q0;
    t->kv_chunks[4 * i + 2] = chunks[i].q1;
    t->kv_chunks[4 * i + 3] = chunks[i].slot;
  }
  build_rot_classes(t);
  return AI_OK;
}

// Index-head rows: one pass over the EXTEND blocks (compute_index_losses,
// attn_layers.py:56-104); `fill` false only counts.
int index_rows(const AiPrepList* l, const int32_t* type, int64_t editable_start, bool fill, int32_t* n_rows_out,
               int64_t* n_keys_out, int64_t* edits, AiIndexRowsOut* out) {
  if (!l || !type) return AI_ERR_NULL;
  if (l->n_blocks < 0 || (l->n_blocks > 0 && (!l->boundary || !l->query_pos || !l->key_pos || !l->attn_mask)))
    return AI_ERR_NULL;
  int32_t nr = 0;
  int64_t nk = 0, lo = 0, hi = 0;
  for (int pass = 0; pass < (fill ? 2 : 1); ++pass) {
    nr = 0;
    nk = 0;
    for (int32_t i = 0; i < l->n_blocks; ++i) {
      if (type[i] != AI_BLOCK_TYPE_EXTEND) continue;
      const int64_t* bd = l->boundary + 4 * (int64_t)i;
      const int64_t s = bd[0], e = bd[1], ks = bd[2], ke = bd[3];
      if (e - s < 2 || ke - ks != e || e > l->n_query || ke > l->n_keys) return AI_ERR_LAYOUT;
      const int64_t ed = e - 1;
      if (!fill && edits) edits[nr / 2] = ed;
      for (int head = 0; head < 2; ++head) {
        const int64_t qi = ed - 1 + head, n = ed + head, qpos = l->query_pos[qi];
        if (fill) {
          int32_t* row = out->rows + 4 * (int64_t)nr;
          row[0] = head;
          row[1] = (int32_t)qi;
          row[2] = (int32_t)n;
          row[3] = (int32_t)nk;
          for (int64_t j = 0; j < n; ++j) {
            const int64_t kp = l->key_pos[ks + j], rel = kp - qpos;
            const bool ok = l->attn_mask[ks + j] && kp >= editable_start && (head == 0 || rel > 0);
            if (pass == 0) {
              if (ok) {
                lo = std::min(lo, rel);
                hi = std::max(hi, rel);
              }
            } else {
              const int64_t r = std::min(std::max(rel - lo, (int64_t)0), hi - lo);
              out->key_rows[nk + j] = (int32_t)r;
              out->key_ok[nk + j] = ok ? 1 : 0;
            }
          }
        }
        ++nr;
        nk += n;
        if (nk > INT32_MAX) return AI_ERR_LAYOUT;
      }
    }
  }
  if (n_rows_out) *n_rows_out = nr;
  if (n_keys_out) *n_keys_out = nk;
  if (fill) {
    out->rel_lo = lo;
    out->rel_hi = hi;
  }
  return AI_OK;
}

}  // namespace

extern "C" {

int ai_attn_positions_from_ops_sizes(const int64_t* ops, int32_t n_ops, int32_t* n_blocks, int64_t* n_query,
                                     int64_t* n_keys) {
  if (!ops || !n_blocks || !n_query || !n_keys) return AI_ERR_NULL;
  return replay_ops(reinterpret_cast<const Op*>(ops), n_ops, nullptr, n_query, n_blocks, n_keys);
}

int ai_attn_positions_from_ops(const int64_t* ops, int32_t n_ops, int64_t* boundary, int64_t* query_pos,
                               int64_t* key_pos, uint8_t* attn_mask, uint8_t* abs_mask, int32_t* block_type) {
  if (!ops || !boundary || !query_pos || !key_pos || !attn_mask || !abs_mask) return AI_ERR_NULL;
  std::vector<PushedBlock> blocks;
  int64_t T = 0, nk = 0;
  int32_t nb = 0;
  int rc = replay_ops(reinterpret_cast<const Op*>(ops), n_ops, &blocks, &T, &nb, &nk);
  if (rc != AI_OK) return rc;
  int64_t kcum = 0, qcum = 0;
  for (int32_t i = 0; i < nb; ++i) {
    const PushedBlock& b = blocks[(size_t)i];
    boundary[4 * (int64_t)i] = b.start;
    boundary[4 * (int64_t)i + 1] = b.end;
    boundary[4 * (int64_t)i + 2] = kcum;
    boundary[4 * (int64_t)i + 3] = kcum + b.end;
    if (block_type) block_type[i] = b.type;
    std::memcpy(key_pos + kcum, b.key_pos.data(), sizeof(int64_t) * (size_t)b.end);
    std::memcpy(attn_mask + kcum, b.attn.data(), (size_t)b.end);
    std::memcpy(abs_mask + kcum, b.abs.data(), (size_t)b.end);
    std::memcpy(query_pos + qcum, b.query_pos.data(), sizeof(int64_t) * b.query_pos.size());
    kcum += b.end;
    qcum += (int64_t)b.query_pos.size();
  }
  return AI_OK;
}

int ai_attn_prep_sizes(const AiPrepList* lists, int32_t n_lists, const int32_t* list_of_row, int32_t batch,
                       int32_t seq_len, int32_t fwd_tile, int32_t kv_tile, AiPrepSizes* sizes) {
  if (!sizes) return AI_ERR_NULL;
  Tables t;
  int rc = build(lists, n_lists, list_of_row, batch, seq_len, fwd_tile, kv_tile, &t);
  if (rc != AI_OK) return rc;
  sizes->n_blocks = (int32_t)(t.blocks.size() / AI_BLOCK_FIELDS);
  sizes->n_fwd_items = (int32_t)(t.fwd_items.size() / 4);
  sizes->n_kv_items = (int32_t)(t.kv_items.size() / 4);
  sizes->n_kv_chunks = (int32_t)(t.kv_chunks.size() / 4);
  sizes->n_kv_reduce = (int32_t)(t.kv_reduce.size() / 4);
  sizes->n_chunk_cls = (int32_t)t.chunk_cls.size();
  sizes->n_rot_classes = (int32_t)(t.rot_classes.size() / 2);
  sizes->n_keys = (int64_t)t.key_info.size();
  sizes->p_min = t.p_min;
  sizes->p_max = t.p_max;
  return AI_OK;
}

int ai_attn_prep(const AiPrepList* lists, int32_t n_lists, const int32_t* list_of_row, int32_t batch,
                 int32_t seq_len, int32_t fwd_tile, int32_t kv_tile, AiPrepTables* out) {
  if (!out || !out->blocks || !out->row_blocks || !out->row_cov || !out->key_info || !out->q_pos || !out->k_own ||
      !out->fwd_items || !out->kv_items || !out->kv_chunks)
    return AI_ERR_NULL;
  Tables t;
  int rc = build(lists, n_lists, list_of_row, batch, seq_len, fwd_tile, kv_tile, &t);
  if (rc != AI_OK) return rc;
  auto put = [](int32_t* dst, const std::vector<int32_t>& v) {
    if (!v.empty()) std::memcpy(dst, v.data(), sizeof(int32_t) * v.size());
  };
  put(out->blocks, t.blocks);
  put(out->row_blocks, t.row_blocks);
  put(out->row_cov, t.row_cov);
  if (!t.key_info.empty()) std::memcpy(out->key_info, t.key_info.data(), sizeof(uint32_t) * t.key_info.size());
  put(out->q_pos, t.q_pos);
  put(out->k_own, t.k_own);
  put(out->fwd_items, t.fwd_items);
  put(out->kv_items, t.kv_items);
  put(out->kv_chunks, t.kv_chunks);
  if (!t.kv_reduce.empty()) {
    if (!out->kv_reduce) return AI_ERR_NULL;
    put(out->kv_reduce, t.kv_reduce);
  }
  if (!out->blk_cls) return AI_ERR_NULL;
  put(out->blk_cls, t.blk_cls);
  if (!t.chunk_cls.empty()) {
    if (!out->chunk_cls || !out->rot_classes) return AI_ERR_NULL;
    put(out->chunk_cls, t.chunk_cls);
    put(out->rot_classes, t.rot_classes);
  }
  out->n_kv_partials = t.n_kv_partials;
  out->kv_cost_max = t.kv_cost_max;
  out->kv_cost_total = t.kv_cost_total;
  out->n_fwd_abs_items = t.n_fwd_abs;
  out->n_fwd_short_items = t.n_fwd_short;
  out->n_fwd_abs_short_items = t.n_fwd_abs_short;
  out->n_kv_abs_items = t.n_kv_abs;
  out->all_rows_owned = t.all_owned ? 1 : 0;
  out->pairs_per_head = t.pairs;
  return AI_OK;
}

int ai_index_rows_sizes(const AiPrepList* list, const int32_t* block_type, int32_t* n_rows, int64_t* n_keys,
                        int64_t* edits) {
  if (!n_rows || !n_keys) return AI_ERR_NULL;
  return index_rows(list, block_type, 0, false, n_rows, n_keys, edits, nullptr);
}

int ai_index_rows(const AiPrepList* list, const int32_t* block_type, int64_t editable_start, AiIndexRowsOut* out) {
  if (!out || !out->rows || !out->key_rows || !out->key_ok) return AI_ERR_NULL;
  return index_rows(list, block_type, editable_start, true, nullptr, nullptr, nullptr, out);
}

}  // extern "C"
