// bpe.cpp -- host BPE encode/decode over the chip's tokenizer ROMs.
//
// Same results as the reference tokenizer (_tape_runner.c:998-1397):
//   * encode: BOS first; special-token strings (all specials but BOS) are
//     matched greedily, longest first, and emitted as their IDs; the text
//     between them becomes metaspace words ("▁" prepended to the first
//     segment, every space turned into "▁", words split before each "▁"),
//     each word is split into UTF-8 characters looked up in the vocab hash
//     (FNV-1a, linear probing), with <0xHH> byte tokens as fallback, and
//     merged by repeatedly applying the lowest-ranked merge present in the
//     word (leftmost pair on ties) to every non-overlapping occurrence;
//   * decode: concatenate the pieces of non-special in-range IDs, turn "▁"
//     into spaces (optionally dropping the first), then replace "<0xHH>"
//     sequences by their byte.
// The merge search uses a hash map from (a, b) to the lowest rank instead of
// scanning the merge table per pair; it picks the same merge.
// One deliberate difference: a multi-byte UTF-8 lead byte cut off by the end
// of the input is looked up as the bytes that exist (the reference reads past
// its buffer there).
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "tape_runner.h"

namespace {

const uint8_t kMeta[3] = {0xE2, 0x96, 0x81};  // "▁" U+2581

inline bool meta_at(const uint8_t *b, int pos, int len) {
    return pos + 2 < len && b[pos] == kMeta[0] && b[pos + 1] == kMeta[1] &&
           b[pos + 2] == kMeta[2];
}

inline int utf8_len(uint8_t lead) {
    if (lead < 0x80) return 1;
    if ((lead & 0xE0) == 0xC0) return 2;
    if ((lead & 0xF0) == 0xE0) return 3;
    if ((lead & 0xF8) == 0xF0) return 4;
    return 1;
}

inline uint32_t fnv1a32(const uint8_t *p, int n) {
    uint32_t h = 2166136261u;
    for (int i = 0; i < n; i++) h = (h ^ p[i]) * 16777619u;
    return h;
}

struct Roms {
    const uint8_t *keys;
    const int32_t *vals;
    const int32_t *lens;
    int table, max_len;

    int lookup(const uint8_t *p, int n) const {
        if (table == 0 || n > max_len) return -1;
        int slot = (int)(fnv1a32(p, n) % (uint32_t)table);
        for (int probe = 0; probe < table; probe++) {
            int sl = lens[slot];
            if (sl == 0) return -1;
            if (sl == n && memcmp(keys + (size_t)slot * max_len, p, n) == 0) return vals[slot];
            slot = (slot + 1) % table;
        }
        return -1;
    }
};

struct MergeTable {
    std::unordered_map<uint64_t, int> rank;   // (a, b) -> lowest rank
    const int32_t *result = nullptr;
    MergeTable(const int32_t *a, const int32_t *b, const int32_t *r, int n) : result(r) {
        rank.reserve((size_t)n * 2 + 1);
        for (int i = 0; i < n; i++) {
            uint64_t k = ((uint64_t)(uint32_t)a[i] << 32) | (uint32_t)b[i];
            rank.emplace(k, i);   // keeps the first (lowest) rank
        }
    }
    int find(int a, int b) const {
        auto it = rank.find(((uint64_t)(uint32_t)a << 32) | (uint32_t)b);
        return it == rank.end() ? -1 : it->second;
    }
};

// One word (metaspace-delimited) to token IDs.
void encode_word(const uint8_t *t, int w0, int w1, const Roms &roms, const MergeTable &mt,
                 std::vector<int> &ids) {
    ids.clear();
    int cpos = w0;
    while (cpos < w1) {
        int clen = meta_at(t, cpos, w1) ? 3 : utf8_len(t[cpos]);
        if (cpos + clen > w1) clen = w1 - cpos;
        int id = roms.lookup(t + cpos, clen);
        if (id >= 0) {
            ids.push_back(id);
        } else {
            for (int b = 0; b < clen; b++) {
                char hex[8];
                int hl = snprintf(hex, sizeof hex, "<0x%02X>", t[cpos + b]);
                int fb = roms.lookup((const uint8_t *)hex, hl);
                if (fb >= 0) ids.push_back(fb);
            }
        }
        cpos += clen;
    }
    while (ids.size() > 1) {
        int best = -1, ba = 0, bb = 0;
        for (size_t i = 0; i + 1 < ids.size(); i++) {
            int r = mt.find(ids[i], ids[i + 1]);
            if (r >= 0 && (best < 0 || r < best)) {
                best = r;
                ba = ids[i];
                bb = ids[i + 1];
            }
        }
        if (best < 0) break;
        int res = mt.result[best];
        size_t w = 0;
        for (size_t i = 0; i < ids.size();) {
            if (i + 1 < ids.size() && ids[i] == ba && ids[i + 1] == bb) {
                ids[w++] = res;
                i += 2;
            } else {
                ids[w++] = ids[i++];
            }
        }
        ids.resize(w);
    }
}

int encode_segment(const uint8_t *raw, int n, bool prepend, int max_tokens, const Roms &roms,
                   const MergeTable &mt, int32_t *out) {
    if (n <= 0 || max_tokens <= 0) return 0;
    std::vector<uint8_t> t;
    t.reserve((size_t)n * 3 + 3);
    if (prepend) t.insert(t.end(), kMeta, kMeta + 3);
    for (int i = 0; i < n; i++) {
        if (raw[i] == ' ')
            t.insert(t.end(), kMeta, kMeta + 3);
        else
            t.push_back(raw[i]);
    }
    int tl = (int)t.size();
    int emitted = 0;
    std::vector<int> ids;
    int ws = 0;
    while (ws < tl) {
        int we = ws;
        if (meta_at(t.data(), we, tl)) we += 3;
        while (we < tl && !meta_at(t.data(), we, tl)) we += utf8_len(t[we]);
        if (we > tl) we = tl;
        if (we <= ws) {
            ws = we + 1;
            continue;
        }
        encode_word(t.data(), ws, we, roms, mt, ids);
        for (size_t i = 0; i < ids.size() && emitted < max_tokens; i++) out[emitted++] = ids[i];
        ws = we;
    }
    return emitted;
}

inline int hexval(uint8_t c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    return 0;
}

}  // namespace

extern "C" int bpe_encode(const uint8_t *raw_bytes, int raw_len, const uint8_t *hash_keys,
                          const int32_t *hash_vals, const int32_t *hash_lens, int table_size,
                          int max_piece_len, const int32_t *merge_a, const int32_t *merge_b,
                          const int32_t *merge_result, int num_merges, int bos_token_id,
                          int max_tokens, const uint8_t *id_to_bytes,
                          const int32_t *id_to_offsets, const int32_t *special_ids,
                          int num_special, int vocab_size, int32_t *out_ids) {
    int n = 0;
    out_ids[n++] = bos_token_id;
    if (raw_len <= 0) return n;
    Roms roms{hash_keys, hash_vals, hash_lens, table_size, max_piece_len};
    MergeTable mt(merge_a, merge_b, merge_result, num_merges);
    struct Sp {
        const uint8_t *p;
        int n, id;
    };
    std::vector<Sp> sp;
    if (id_to_bytes && id_to_offsets && special_ids) {
        for (int s = 0; s < num_special; s++) {
            int id = special_ids[s];
            if (id == bos_token_id || id < 0 || id >= vocab_size) continue;
            int len = id_to_offsets[2 * id + 1];
            if (len <= 0) continue;
            sp.push_back({id_to_bytes + id_to_offsets[2 * id], len, id});
        }
    }
    auto special_at = [&](int pos, bool longest) -> int {
        int best = -1, bl = 0;
        for (size_t s = 0; s < sp.size(); s++) {
            if (pos + sp[s].n > raw_len) continue;
            if (sp[s].n > bl && memcmp(raw_bytes + pos, sp[s].p, sp[s].n) == 0) {
                best = (int)s;
                bl = sp[s].n;
                if (!longest) break;
            }
        }
        return best;
    };
    int pos = 0;
    bool first = true;
    while (pos < raw_len && n < max_tokens) {
        int m = special_at(pos, true);
        if (m >= 0) {
            out_ids[n++] = sp[m].id;
            pos += sp[m].n;
            first = false;
            continue;
        }
        int end = pos + 1;
        while (end < raw_len && special_at(end, false) < 0) end++;
        n += encode_segment(raw_bytes + pos, end - pos, first, max_tokens - n, roms, mt,
                            out_ids + n);
        pos = end;
        first = false;
    }
    return n;
}

extern "C" int bpe_decode(const int32_t *token_ids, int num_tokens, const uint8_t *id_to_bytes,
                          const int32_t *id_to_offsets, int vocab_size,
                          const int32_t *special_ids, int num_special, int max_bytes,
                          int skip_leading_space, uint8_t *out_bytes) {
    std::vector<uint8_t> raw;
    raw.reserve((size_t)(max_bytes > 0 ? max_bytes : 0) + 256);
    for (int i = 0; i < num_tokens; i++) {
        int id = token_ids[i];
        bool special = false;
        for (int s = 0; s < num_special && !special; s++) special = id == special_ids[s];
        if (special || id < 0 || id >= vocab_size) continue;
        int off = id_to_offsets[2 * id], len = id_to_offsets[2 * id + 1];
        if (len == 0) continue;
        if ((long long)raw.size() + len < (long long)max_bytes + 256)
            raw.insert(raw.end(), id_to_bytes + off, id_to_bytes + off + len);
    }
    int rl = (int)raw.size(), ol = 0;
    bool skip = skip_leading_space != 0;
    std::vector<uint8_t> spaced;
    spaced.reserve(raw.size());
    for (int i = 0; i < rl && ol < max_bytes;) {
        if (meta_at(raw.data(), i, rl)) {
            if (skip)
                skip = false;
            else {
                spaced.push_back(' ');
                ol++;
            }
            i += 3;
        } else {
            spaced.push_back(raw[i++]);
            ol++;
            skip = false;
        }
    }
    int fl = 0;
    for (int i = 0; i < ol;) {
        if (i + 5 < ol && spaced[i] == '<' && spaced[i + 1] == '0' && spaced[i + 2] == 'x') {
            int j = i + 3;
            while (j < ol && spaced[j] != '>') j++;
            if (j < ol && j - (i + 3) == 2) {
                out_bytes[fl++] = (uint8_t)(hexval(spaced[i + 3]) * 16 + hexval(spaced[i + 4]));
                i = j + 1;
                continue;
            }
        }
        out_bytes[fl++] = spaced[i++];
    }
    return fl;
}
