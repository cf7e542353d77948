// Host planner: turns the step's batch description into the packed int32 plan every layer reads.
//
// Replaces build_attention_metadata and its helpers (src/miniserve/attention/backends.py:80-142).
// The reference sorts short-query rows by context length, pads them into groups under a gather
// cap, and builds int64 index tensors and boolean masks per group; prefill chunks get their own
// slot lists and shifted causal masks.  Here nothing is padded or gathered: each sequence keeps
// its own block table (CSR), and the work is cut into (query tile, KV page range) items:
//   * a sequence with <= 8 new tokens (decode, speculative verify) is one decode tile;
//   * a chunk of 9..64 tokens is one tile for the mma.sync tile kernel;
//   * a chunk of more than 64 tokens is cut into items of two 64-token query tiles (2 x 128 rows)
//     for the tcgen05 tensor-core kernel: groups g and G-1-g of the chunk when no item of the
//     chunk is split (equal causal work per item), else adjacent groups, whose page ranges are
//     split in whole 128-key blocks.  Tensor-core records carry tile A as (tok0, n_q) and tile B
//     as fields 6 and 7 (first token, count; count 0 for no tile B);
//   * a tile's visible pages, ceil((num_cached + tok0 + n_q) / 16), are split into near-equal
//     ranges of at most `pages_per_split` pages; split tiles get partial rows in the workspace
//     and a combine record.
//   * a run of >= 16 consecutive decode / verify rows, contiguous in the batch, whose block tables
//     begin with the same >= 16 cached blocks is a cascade group: the shared prefix is attended
//     once by tensor-core items over all the group's query tokens (a virtual sequence record
//     after the real ones, run first), and each row's remaining pages by an unsplit decode item
//     whose epilogue merges the prefix partials.
// Items are ordered longest first so the hardware block scheduler fills the tail with short ones.
#include <algorithm>
#include <climits>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/msattn.h"

namespace ms_host {
void set_error(const std::string& msg);
}

namespace {

constexpr int kRec = 8;
constexpr int kDecodeMaxTokens = 8;  // backends.py:32 SHORT_QUERY: the batched (short) path
constexpr int kTileTokens = 64;      // longest chunk of the mma.sync tile kernel (128 rows)
constexpr int kTcTokens = 128;       // query tokens per tensor-core work item (2 x 128 rows)
// Automatic split of decode / small-tile items: the smallest split (a multiple of 8 pages, at
// least kMinSplitPages) whose items fit one resident wave of CTAs -- kDecodeCtasPerSm per SM,
// kTcAssumedKvHeads CTAs per item -- or no split (up to kMaxSplitPages) when the rows alone
// exceed a wave.  Measured on 1x B200 (us per attention call): 1 row of 32K tokens 36.4 with
// 64-page splits vs 50.2 with 32; 4 x 16K 47.6 (128) vs 64.5 (32); config 3's 48 decode rows
// 41.0 unsplit vs 46.5 (32).  Splits that leave a thin second wave are the worst case.  Small
// batches far below a wave split down to 8 pages: 8 rows of U[1, 512] context 12.5 -> 9.9 us per
// layer-step (one page range per CTA streams at only a few tens of GB/s); 16 rows of 1000
// tokens 20.8 -> 14.7 us; 8 verify rows of 5 over 2000 22.9 -> 16.4 us.
constexpr int kDecodeCtasPerSm = 2;
constexpr int kMinSplitPages = 8;
constexpr int kMaxSplitPages = 512;
constexpr int kTcBlockPages = 8;     // 128-key blocks of the tensor-core kernel
constexpr int kTcMinSplitPages = 32; // forced splits: tensor-core items cover at least 4 blocks
// Automatic tensor-core plan.  The planner does not see the head count; it sizes work for
// kTcAssumedKvHeads CTAs per item (Qwen3-0.6B's 8 KV heads), which only affects speed.
//  * When the unsplit items already fill one wave (items x heads >= SMs), they stay whole and
//    adjacent; longest-first order packs the waves.
//  * Otherwise key ranges are split so that about one wave of CTAs results, but never below
//    kTcAutoMinSplitPages (each CTA's start-up is worth about two blocks of work), and a chunk
//    that needs no split pairs its 64-token groups zig-zag so the items of the wave cost alike.
constexpr int kTcAssumedKvHeads = 8;
constexpr int kTcAutoMinSplitPages = 128;
// Cascade (shared-prefix) attention: a run of consecutive decode / verify rows, contiguous in the
// batch, whose block tables start with the same whole cached blocks attends that prefix once, as
// one dense tensor-core problem over all the run's query tokens, instead of once per row.
constexpr int kCascadeMinRows = 16;
constexpr int kCascadeMinPages = 16;

struct Item {
  int seq, tok0, n_q, pb, pe, part_row;
  // Fields 6 and 7.  Tensor-core items: tile B's first token and token count.  Decode items of
  // cascade rows: the first shared-prefix partial row to merge, and 1.
  int tok_b = 0, n_b = 0;
};

int64_t round4(int64_t x) { return (x + 3) & ~int64_t(3); }

}  // namespace

extern "C" int64_t ms_plan_capacity(int32_t num_seqs, int32_t num_tokens,
                                    int64_t total_table_entries) {
  // Every item covers at least one page and every tile at least one query token, so the number
  // of items is bounded by tiles * pages; a looser closed form is enough: one decode/tile item per
  // 16 table entries plus one per tile, plus as many combine records.
  const int64_t tiles = static_cast<int64_t>(num_seqs) + num_tokens / kTileTokens + 1;
  const int64_t items = tiles + total_table_entries;
  // Cascade groups add one sequence record each (at most num_seqs / kCascadeMinRows), tensor-core
  // items over their query tokens (at most one per 64 tokens plus one per group) and one combine
  // record per row (within the combine bound above).
  const int64_t groups = static_cast<int64_t>(num_seqs) / kCascadeMinRows + 1;
  return round4(static_cast<int64_t>(num_seqs) * kRec) + round4(total_table_entries) +
         3 * round4(items * kRec) + round4(tiles * kRec) + round4(groups * kRec) +
         round4((num_tokens / kTileTokens + groups) * kRec) + 16;
}

extern "C" int ms_plan_build(int32_t num_seqs, const int32_t* flat_start, const int32_t* num_new,
                             const int32_t* num_cached, const int64_t* table_offsets,
                             const int32_t* tables, int32_t num_tokens, int32_t block_size,
                             int32_t num_sms, int32_t pages_per_split, int32_t* out,
                             int64_t out_capacity, MsPlanInfo* info) {
  if (info == nullptr || out == nullptr) {
    ms_host::set_error("ms_plan_build: null output");
    return MS_ERR_ARG;
  }
  std::memset(info, 0, sizeof(*info));
  if (num_seqs < 0 || num_tokens < 0 || block_size != 16 || num_sms <= 0 || pages_per_split < 0) {
    ms_host::set_error("ms_plan_build: bad sizes (block_size must be 16, num_sms > 0)");
    return MS_ERR_ARG;
  }
  if (num_seqs > 0 && (flat_start == nullptr || num_new == nullptr || num_cached == nullptr ||
                       table_offsets == nullptr)) {
    ms_host::set_error("ms_plan_build: null batch arrays");
    return MS_ERR_ARG;
  }
  const int64_t total_entries = num_seqs > 0 ? table_offsets[num_seqs] : 0;
  if (total_entries > 0 && tables == nullptr) {
    ms_host::set_error("ms_plan_build: null block tables");
    return MS_ERR_ARG;
  }
  if (total_entries >= (int64_t(1) << 31)) {
    ms_host::set_error("ms_plan_build: block tables exceed 2^31 entries");
    return MS_ERR_ARG;
  }

  // Validate sequences and cut query tiles.
  std::vector<Item> tiles;
  tiles.reserve(num_seqs);
  int64_t total_pages = 0;
  for (int i = 0; i < num_seqs; ++i) {
    const int64_t n = num_new[i], c = num_cached[i], f = flat_start[i];
    const int64_t tlen = table_offsets[i + 1] - table_offsets[i];
    if (n < 1 || c < 0 || f < 0 || f + n > num_tokens || tlen < 0) {
      ms_host::set_error("ms_plan_build: sequence " + std::to_string(i) +
                         " has an invalid flat_start/num_new/num_cached");
      return MS_ERR_PLAN;
    }
    const int64_t ctx = c + n;
    if (ctx >= (int64_t(1) << 30)) {
      ms_host::set_error("ms_plan_build: context too long");
      return MS_ERR_PLAN;
    }
    if (tlen * block_size < ctx) {
      ms_host::set_error("ms_plan_build: sequence " + std::to_string(i) + " needs " +
                         std::to_string((ctx + block_size - 1) / block_size) +
                         " blocks but its table has " + std::to_string(tlen));
      return MS_ERR_PLAN;
    }
    const int step = n <= kDecodeMaxTokens ? kDecodeMaxTokens : (n <= kTileTokens ? kTileTokens : kTcTokens);
    for (int64_t t0 = 0; t0 < n; t0 += step) {
      const int nq = static_cast<int>(std::min<int64_t>(step, n - t0));
      const int pages = static_cast<int>((c + t0 + nq + block_size - 1) / block_size);
      tiles.push_back({i, static_cast<int>(t0), nq, 0, pages, -1});
      total_pages += pages;
    }
  }

  // Cascade groups: runs of decode / verify rows, consecutive in the batch, whose tables begin
  // with the same kCascadeMinPages or more whole cached blocks.  cascade_pages[i] is the shared
  // prefix (in pages) of row i's group, 0 outside groups.
  struct Group {
    int first, last, pages, tokens;
  };
  std::vector<Group> groups;
  std::vector<int> cascade_pages(num_seqs, 0);
  {
    auto eligible = [&](int i) {
      return num_new[i] <= kDecodeMaxTokens &&
             num_cached[i] >= static_cast<int64_t>(kCascadeMinPages) * block_size;
    };
    int i = 0;
    while (i < num_seqs) {
      if (!eligible(i)) {
        ++i;
        continue;
      }
      const int32_t* ti = tables + table_offsets[i];
      int64_t shared = std::min<int64_t>(num_cached[i] / block_size,
                                         table_offsets[i + 1] - table_offsets[i]);
      int64_t tokens = num_new[i];
      int j = i + 1;
      while (j < num_seqs && eligible(j) &&
             static_cast<int64_t>(flat_start[j]) == static_cast<int64_t>(flat_start[j - 1]) + num_new[j - 1]) {
        const int32_t* tj = tables + table_offsets[j];
        const int64_t cap = std::min<int64_t>(shared, num_cached[j] / block_size);
        int64_t l = 0;
        while (l < cap && tj[l] == ti[l]) ++l;
        if (l < kCascadeMinPages) break;
        shared = l;
        tokens += num_new[j];
        ++j;
      }
      if (j - i >= kCascadeMinRows && tokens > kTileTokens) {
        groups.push_back({i, j, static_cast<int>(shared), static_cast<int>(tokens)});
        for (int k = i; k < j; ++k) {
          cascade_pages[k] = static_cast<int>(shared);
        }
        i = j;
      } else {
        ++i;
      }
    }
  }

  // Split size for the bandwidth-bound kernels (see kDecodeCtasPerSm).
  int split = pages_per_split;
  if (split == 0) {
    const int64_t target_items =
        std::max<int64_t>(1, static_cast<int64_t>(num_sms) * kDecodeCtasPerSm / kTcAssumedKvHeads);
    auto items_at = [&](int p) {
      int64_t items = 0;
      for (const Item& t : tiles)
        if (num_new[t.seq] <= kTileTokens && cascade_pages[t.seq] == 0) items += (t.pe + p - 1) / p;
      return items;
    };
    // items_at() does not grow with the split, so the smallest fitting split is found by
    // bisection over multiples of 8 pages.
    int lo = kMinSplitPages / 8, hi = kMaxSplitPages / 8;
    bool has_tc = !groups.empty();
    for (const Item& t : tiles) has_tc = has_tc || num_new[t.seq] > kTileTokens;
    if (items_at(hi * 8) > target_items) {
      // The rows alone exceed a wave.  Longest-first order then packs the waves, except that an
      // item longer than the pages per item-slot (all pages / a wave's items) outlasts them:
      // without tensor-core work, split just those, into pieces of about that size (60 rows of
      // 100 tokens + 4 of 4000: 77.0 -> 25.2 us).  Beside tensor-core work the decode launch
      // overlaps it on a second stream and a combine pass would wait for both: config 3 measured
      // 71.2 us per layer-step unsplit against 77.3 (96-page pieces), 73.2 (64) and 77.4 (48),
      // so they stay whole there.
      split = kMaxSplitPages;
      if (!has_tc) {
        int64_t pages = 0;
        for (const Item& t : tiles)
          if (num_new[t.seq] <= kTileTokens && cascade_pages[t.seq] == 0) pages += t.pe;
        const int64_t per_slot = (pages + target_items - 1) / target_items;
        split = static_cast<int>(std::min<int64_t>(
            kMaxSplitPages, std::max<int64_t>(kMinSplitPages, (per_slot + 7) / 8 * 8)));
      }
    } else {
      while (lo < hi) {
        const int mid = (lo + hi) / 2;
        if (items_at(mid * 8) <= target_items) hi = mid; else lo = mid + 1;
      }
      split = lo * 8;
    }
  }

  std::vector<Item> dec, til, tcv, comb;
  int64_t part_rows = 0;
  int64_t n_tc_tiles = 0, tc_pages = 0;
  for (const Item& t : tiles) {
    if (num_new[t.seq] > kTileTokens) {
      ++n_tc_tiles;
      tc_pages += t.pe;
    }
  }
  auto round_blocks = [](int64_t p) { return (p + kTcBlockPages - 1) / kTcBlockPages * kTcBlockPages; };
  int64_t tc_split64;
  if (pages_per_split > 0) {
    tc_split64 = std::max<int64_t>(kTcMinSplitPages, round_blocks(pages_per_split));
  } else if (n_tc_tiles * kTcAssumedKvHeads >= num_sms) {
    tc_split64 = int64_t(1) << 30;
  } else {
    // The smallest split (whole 128-key blocks, at least kTcAutoMinSplitPages) whose items fit
    // one wave, one CTA per SM.  The work-per-CTA estimate alone is not enough: every tile's
    // split count rounds up, which can leave a thin second wave (8 tiles over 8192 cached tokens:
    // 240 pages gave 24 items, 192 CTAs).  The CTA count does not grow with the split, so the
    // split is found by bisection; at the longest tile's page count every tile is one item and
    // the items fit (this branch has fewer tiles x heads than SMs).
    auto tc_ctas_at = [&](int64_t p) {
      int64_t items = 0;
      for (const Item& t : tiles)
        if (num_new[t.seq] > kTileTokens && cascade_pages[t.seq] == 0) items += (t.pe + p - 1) / p;
      return items * kTcAssumedKvHeads;
    };
    int64_t max_pe = 0;
    for (const Item& t : tiles)
      if (num_new[t.seq] > kTileTokens) max_pe = std::max<int64_t>(max_pe, t.pe);
    const int64_t per_cta = (tc_pages * kTcAssumedKvHeads + num_sms - 1) / std::max(num_sms, 1);
    int64_t lo = std::max<int64_t>(kTcAutoMinSplitPages, round_blocks(per_cta)) / kTcBlockPages;
    int64_t hi = std::max<int64_t>(lo, round_blocks(max_pe) / kTcBlockPages);
    while (lo < hi) {
      const int64_t mid = (lo + hi) / 2;
      if (tc_ctas_at(mid * kTcBlockPages) <= num_sms) hi = mid; else lo = mid + 1;
    }
    tc_split64 = lo * kTcBlockPages;
  }
  const int tc_split = static_cast<int>(std::min<int64_t>(tc_split64, int64_t(1) << 30));
  const bool tc_zigzag = pages_per_split > 0 || n_tc_tiles * kTcAssumedKvHeads < num_sms;
  for (const Item& t : tiles) {
    const int pages = t.pe;
    const int nn = num_new[t.seq];
    const bool is_tc = nn > kTileTokens;
    if (cascade_pages[t.seq] > 0) continue;  // planned with its cascade group below
    if (is_tc) {
      // A chunk none of whose items is split pairs its 64-token groups zig-zag: tile A = group
      // g, tile B = group G-1-g.  Causal work grows with the group index, so every pair costs
      // about the same and the slowest item no longer sets the kernel's time.
      const int64_t c = num_cached[t.seq];
      const int64_t chunk_pages = (c + nn + block_size - 1) / block_size;
      if (tc_zigzag && chunk_pages <= tc_split) {
        if (t.tok0 != 0) continue;  // the whole chunk is emitted with its first tile
        const int groups = (nn + kTileTokens - 1) / kTileTokens;
        for (int g = 0; g < (groups + 1) / 2; ++g) {
          const int h = groups - 1 - g;
          Item it{t.seq, g * kTileTokens, std::min(kTileTokens, nn - g * kTileTokens), 0, 0, -1};
          if (h > g) {
            it.tok_b = h * kTileTokens;
            it.n_b = std::min(kTileTokens, nn - it.tok_b);
          }
          const int64_t last = h > g ? it.tok_b + it.n_b : it.tok0 + it.n_q;
          it.pe = static_cast<int>((c + last + block_size - 1) / block_size);
          tcv.push_back(it);
        }
        continue;
      }
    }
    const int sp = is_tc ? tc_split : split;
    const int ns = (pages + sp - 1) / sp;
    std::vector<Item>& dst = nn <= kDecodeMaxTokens ? dec : (is_tc ? tcv : til);
    // Tensor-core items that are split keep their two tiles adjacent (A = tokens tok0..+63, B =
    // the next 64), so the partial rows of the item are its tokens in order for the combine.
    const int n_a = is_tc ? std::min(kTileTokens, t.n_q) : t.n_q;
    const int tok_b = is_tc ? t.tok0 + kTileTokens : 0;
    const int n_b = is_tc ? std::max(0, t.n_q - kTileTokens) : 0;
    if (ns <= 1) {
      dst.push_back({t.seq, t.tok0, n_a, 0, pages, -1, tok_b, n_b});
      continue;
    }
    const int rows = 2 * t.n_q;
    if (part_rows + static_cast<int64_t>(ns) * rows >= (int64_t(1) << 31)) {
      ms_host::set_error("ms_plan_build: too many partial rows");
      return MS_ERR_PLAN;
    }
    // Near-equal ranges; tensor-core ranges stay whole 128-key blocks except the last.
    const int unit = is_tc ? kTcBlockPages : 1;
    const int units = (pages + unit - 1) / unit;
    const int base = units / ns, rem = units % ns;
    int pb = 0;
    for (int s = 0; s < ns; ++s) {
      const int len = std::min(pages - pb, (base + (s < rem ? 1 : 0)) * unit);
      dst.push_back({t.seq, t.tok0, n_a, pb, pb + len,
                     static_cast<int>(part_rows + static_cast<int64_t>(s) * rows), tok_b, n_b});
      pb += len;
    }
    comb.push_back({t.seq, t.tok0, t.n_q, static_cast<int>(part_rows), ns, 0});
    part_rows += static_cast<int64_t>(ns) * rows;
  }
  // Cascade groups.  The shared prefix is attended once by tensor-core items over a virtual
  // sequence (record num_seqs + g): the group's query tokens, contiguous in the batch, with the
  // prefix as their cached context, so every prefix key is visible to every query.  Its items
  // write partial rows for all the group's tokens (the tensor-core kernel runs first); each row
  // then attends its own pages after the prefix with an unsplit decode item whose epilogue
  // merges the row's prefix partials (fields 6 and 7: first partial row, 1).
  for (size_t g = 0; g < groups.size(); ++g) {
    const Group& G = groups[g];
    if (part_rows + 2 * static_cast<int64_t>(G.tokens) >= (int64_t(1) << 31)) {
      ms_host::set_error("ms_plan_build: too many partial rows");
      return MS_ERR_PLAN;
    }
    const int vseq = num_seqs + static_cast<int>(g);
    const int64_t prefix_base = part_rows;
    part_rows += 2 * static_cast<int64_t>(G.tokens);
    for (int tok = 0; tok < G.tokens; tok += kTcTokens) {
      const int nq = std::min(kTcTokens, G.tokens - tok);
      tcv.push_back({vseq, tok, std::min(kTileTokens, nq), 0, G.pages,
                     static_cast<int>(prefix_base + 2 * tok), tok + kTileTokens,
                     std::max(0, nq - kTileTokens)});
    }
    for (int k = G.first; k < G.last; ++k) {
      const int n = num_new[k];
      const int pages = static_cast<int>((static_cast<int64_t>(num_cached[k]) + n + block_size - 1) / block_size);
      const int64_t prefix_row = prefix_base + 2 * (static_cast<int64_t>(flat_start[k]) - flat_start[G.first]);
      // Own pages, merged with the prefix partial in the decode kernel's epilogue (field 7 = 1).
      dec.push_back({k, 0, n, G.pages, pages, -1, static_cast<int>(prefix_row), 1});
    }
  }

  auto longest_first = [](const Item& x, const Item& y) { return (x.pe - x.pb) > (y.pe - y.pb); };
  std::stable_sort(dec.begin(), dec.end(), longest_first);
  std::stable_sort(til.begin(), til.end(), longest_first);
  std::stable_sort(tcv.begin(), tcv.end(), longest_first);

  const int64_t off_seqs = 0;
  const int64_t n_seq_records = static_cast<int64_t>(num_seqs) + static_cast<int64_t>(groups.size());
  const int64_t off_tables = round4(off_seqs + n_seq_records * kRec);
  const int64_t off_decode = round4(off_tables + total_entries);
  const int64_t off_tile = round4(off_decode + static_cast<int64_t>(dec.size()) * kRec);
  const int64_t off_tc = round4(off_tile + static_cast<int64_t>(til.size()) * kRec);
  const int64_t off_combine = round4(off_tc + static_cast<int64_t>(tcv.size()) * kRec);
  const int64_t total = round4(off_combine + static_cast<int64_t>(comb.size()) * kRec);
  if (total > out_capacity) {
    ms_host::set_error("ms_plan_build: output buffer holds " + std::to_string(out_capacity) +
                       " ints, plan needs " + std::to_string(total));
    return MS_ERR_CAPACITY;
  }
  if (total >= (int64_t(1) << 31)) {
    ms_host::set_error("ms_plan_build: plan larger than 2^31 ints");
    return MS_ERR_PLAN;
  }
  std::memset(out, 0, sizeof(int32_t) * total);
  for (int i = 0; i < num_seqs; ++i) {
    int32_t* r = out + off_seqs + static_cast<int64_t>(i) * kRec;
    r[0] = flat_start[i];
    r[1] = num_new[i];
    r[2] = num_cached[i];
    r[3] = num_cached[i] + num_new[i];
    r[4] = static_cast<int32_t>(table_offsets[i]);
    r[5] = static_cast<int32_t>(table_offsets[i + 1] - table_offsets[i]);
  }
  for (size_t g = 0; g < groups.size(); ++g) {
    const Group& G = groups[g];
    int32_t* r = out + off_seqs + (static_cast<int64_t>(num_seqs) + static_cast<int64_t>(g)) * kRec;
    r[0] = flat_start[G.first];
    r[1] = G.tokens;
    r[2] = G.pages * block_size;
    r[3] = G.pages * block_size + G.tokens;
    r[4] = static_cast<int32_t>(table_offsets[G.first]);
    r[5] = G.pages;
  }
  if (total_entries > 0) std::memcpy(out + off_tables, tables, sizeof(int32_t) * total_entries);
  auto put = [&](int64_t off, const std::vector<Item>& v) {
    for (size_t k = 0; k < v.size(); ++k) {
      int32_t* r = out + off + static_cast<int64_t>(k) * kRec;
      r[0] = v[k].seq;
      r[1] = v[k].tok0;
      r[2] = v[k].n_q;
      r[3] = v[k].pb;
      r[4] = v[k].pe;
      r[5] = v[k].part_row;
      r[6] = v[k].tok_b;
      r[7] = v[k].n_b;
    }
  };
  put(off_decode, dec);
  put(off_tile, til);
  put(off_tc, tcv);
  for (size_t k = 0; k < comb.size(); ++k) {
    int32_t* r = out + off_combine + static_cast<int64_t>(k) * kRec;
    r[0] = comb[k].seq;
    r[1] = comb[k].tok0;
    r[2] = comb[k].n_q;
    r[3] = comb[k].pb;
    r[4] = comb[k].pe;
    r[5] = comb[k].part_row;  // split stride in partial rows (0: 2 * n_q)
  }

  info->num_seqs = num_seqs;
  info->num_tokens = num_tokens;
  info->n_decode_items = static_cast<int32_t>(dec.size());
  info->n_tile_items = static_cast<int32_t>(til.size());
  info->n_combine = static_cast<int32_t>(comb.size());
  info->off_seqs = static_cast<int32_t>(off_seqs);
  info->off_tables = static_cast<int32_t>(off_tables);
  info->off_decode = static_cast<int32_t>(off_decode);
  info->off_tile = static_cast<int32_t>(off_tile);
  info->n_tc_items = static_cast<int32_t>(tcv.size());
  info->n_cascade = static_cast<int32_t>(groups.size());
  int64_t decode_pages = 0;
  for (const Item& t : dec) decode_pages += t.pe - t.pb;
  info->decode_pages = static_cast<int32_t>(std::min<int64_t>(decode_pages, INT32_MAX));
  int combine_tokens_max = 0;
  for (const Item& c : comb) combine_tokens_max = std::max(combine_tokens_max, c.n_q);
  info->combine_tokens_max = combine_tokens_max;
  info->off_tc = static_cast<int32_t>(off_tc);
  info->off_combine = static_cast<int32_t>(off_combine);
  info->total_ints = static_cast<int32_t>(total);
  info->pages_per_split = split;
  info->part_rows = part_rows;
  info->total_pages = total_pages;
  // ws_o [part_rows][KVH][128] fp32 then ws_lse [part_rows][KVH]; KVH is not known here, so the
  // size is reported per KV head and scaled by the attention call.
  info->workspace_bytes_per_kv_head = part_rows * (128 + 1) * 4;
  return MS_OK;
}

extern "C" int ms_prepare_step(int32_t num_seqs, const int32_t* num_new, const int32_t* num_cached,
                               const int64_t* table_offsets, const int32_t* tables,
                               int32_t block_size, int32_t* flat_start, int64_t* positions,
                               int64_t* slot_mapping, int64_t capacity_tokens,
                               int32_t* num_tokens) {
  if (num_tokens == nullptr || num_seqs < 0 || block_size <= 0 || capacity_tokens < 0) {
    ms_host::set_error("ms_prepare_step: bad sizes");
    return MS_ERR_ARG;
  }
  *num_tokens = 0;
  if (num_seqs > 0 && (num_new == nullptr || num_cached == nullptr || table_offsets == nullptr ||
                       flat_start == nullptr)) {
    ms_host::set_error("ms_prepare_step: null batch arrays");
    return MS_ERR_ARG;
  }
  int64_t flat = 0;
  for (int i = 0; i < num_seqs; ++i) {
    const int64_t n = num_new[i], c = num_cached[i];
    const int64_t off = table_offsets[i], tlen = table_offsets[i + 1] - off;
    if (n < 1 || c < 0 || tlen < 0 || off < 0) {
      ms_host::set_error("ms_prepare_step: sequence " + std::to_string(i) +
                         " has an invalid num_new/num_cached/table");
      return MS_ERR_ARG;
    }
    if (tlen * block_size < c + n) {
      ms_host::set_error("ms_prepare_step: sequence " + std::to_string(i) + " needs " +
                         std::to_string((c + n + block_size - 1) / block_size) +
                         " blocks but its table has " + std::to_string(tlen));
      return MS_ERR_PLAN;
    }
    if (flat + n > capacity_tokens || flat + n >= (int64_t(1) << 31)) {
      ms_host::set_error("ms_prepare_step: more than " + std::to_string(capacity_tokens) +
                         " tokens scheduled");
      return MS_ERR_CAPACITY;
    }
    if (n > 0 && (positions == nullptr || slot_mapping == nullptr || tables == nullptr)) {
      ms_host::set_error("ms_prepare_step: null output arrays");
      return MS_ERR_ARG;
    }
    flat_start[i] = static_cast<int32_t>(flat);
    const int32_t* table = tables + off;
    for (int64_t p = c; p < c + n; ++p, ++flat) {
      positions[flat] = p;
      slot_mapping[flat] = static_cast<int64_t>(table[p / block_size]) * block_size + p % block_size;
    }
  }
  *num_tokens = static_cast<int32_t>(flat);
  return MS_OK;
}
