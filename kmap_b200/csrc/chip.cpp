// chip.cpp -- chip directory loader (C ABI: kllm_chip_*).
//
// Reads the files the kllm compiler writes (reference kllm_compile.c:1705-1890)
// with the same interpretation as the reference CLI's chip_load
// (kllm.c:152-388):
//   processor.json   integer keys + input_map / output_map slot ids
//                    (kllm.c:157-198; a flat key scan, as there)
//   tables/          embed_table.bin [V][H], rope_cos/sin.bin [S][hd] fp32
//   bpe/             hash ROMs, merges, special ids (BOS = special_ids[1]),
//                    id_to_bytes / id_to_offsets
//   circuit/         tape.bin [n, 276, records], slots.bin [n, {type, ndim,
//                    shape[8]}], const_<slot>.bin, const_<slot>_codebook.bin,
//                    const_<slot>_indices.bin (mapped read-only, not read: the
//                    upload copies it to HBM once)
// and builds the TapeCtx the same way: type 4 -> truth table, type 1 ->
// external const, types 2/3 -> allocated.  Unlike the reference it checks
// every size it relies on and fails with an error message instead of exit().
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <vector>

#include "common.cuh"

using kllm::set_error;

struct kllm_chip {
    TapeCtx *ctx = nullptr;
    int vocab = 0, hidden = 0, layers = 0, n_kv = 0, head_dim = 0, max_seq = 0, eos = -1;
    int embed_slot = -1, cos_slot = -1, sin_slot = -1, logits_slot = -1;
    std::vector<int> kv_in, kv_out;
    std::vector<float> embed, rope_cos, rope_sin;
    std::vector<uint8_t> hash_keys, id_to_bytes;
    std::vector<int32_t> hash_vals, hash_lens, merge_a, merge_b, merge_result, special,
        id_to_offsets;
    int table_size = 0, max_piece_len = 0, bos = 1;
    std::vector<std::vector<float>> fbufs;      // const slots / codebooks
    std::vector<std::vector<uint16_t>> ibufs;   // index matrices (empty ones)
    // index matrices mapped from their files (read by the upload, which
    // copies them to HBM once; the pages never need a second host copy)
    std::vector<std::pair<void *, size_t>> maps;
};

namespace {

bool read_file(const std::string &path, std::vector<uint8_t> &out) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) {
        set_error("cannot open %s", path.c_str());
        return false;
    }
    struct stat st;
    if (fstat(fileno(f), &st) != 0) {
        fclose(f);
        set_error("cannot stat %s", path.c_str());
        return false;
    }
    out.resize((size_t)st.st_size);
    size_t got = out.empty() ? 0 : fread(out.data(), 1, out.size(), f);
    fclose(f);
    if (got != out.size()) {
        set_error("short read of %s", path.c_str());
        return false;
    }
    return true;
}

template <class T>
bool read_array(const std::string &path, std::vector<T> &out, size_t expect = (size_t)-1) {
    std::vector<uint8_t> raw;
    if (!read_file(path, raw)) return false;
    if (raw.size() % sizeof(T)) {
        set_error("%s: size %zu is not a multiple of %zu", path.c_str(), raw.size(), sizeof(T));
        return false;
    }
    if (expect != (size_t)-1 && raw.size() != expect * sizeof(T)) {
        set_error("%s: %zu bytes, expected %zu", path.c_str(), raw.size(), expect * sizeof(T));
        return false;
    }
    out.resize(raw.size() / sizeof(T));
    if (!raw.empty()) memcpy(out.data(), raw.data(), raw.size());
    return true;
}

// Map a file of exactly `expect` bytes read-only; nullptr (error set) otherwise.
const void *map_file(const std::string &path, size_t expect, std::vector<std::pair<void *, size_t>> &maps) {
    const int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        set_error("cannot open %s", path.c_str());
        return nullptr;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || (size_t)st.st_size != expect) {
        close(fd);
        set_error("%s: %lld bytes, expected %zu", path.c_str(), (long long)st.st_size, expect);
        return nullptr;
    }
    void *p = mmap(nullptr, expect, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) {
        set_error("cannot map %s", path.c_str());
        return nullptr;
    }
    madvise(p, expect, MADV_SEQUENTIAL | MADV_WILLNEED);
    maps.push_back({p, expect});
    return p;
}

// Integer after "key": (first occurrence), -1 when absent (kllm.c:31-40).
int json_int(const std::string &j, const std::string &key, size_t from = 0, size_t to = std::string::npos) {
    std::string pat = "\"" + key + "\"";
    size_t p = j.find(pat, from);
    if (p == std::string::npos || (to != std::string::npos && p > to)) return -1;
    p += pat.size();
    while (p < j.size() && (j[p] == ' ' || j[p] == ':' || j[p] == '\t' || j[p] == '\n' || j[p] == '\r'))
        p++;
    return atoi(j.c_str() + p);
}

// Integer of child key inside the "parent": { ... } object (kllm.c:45-63).
int json_nested(const std::string &j, const std::string &parent, const std::string &child) {
    size_t p = j.find("\"" + parent + "\"");
    if (p == std::string::npos) return -1;
    size_t b = j.find('{', p);
    if (b == std::string::npos) return -1;
    size_t e = j.find('}', b);
    if (e == std::string::npos) return -1;
    return json_int(j, child, b, e);
}

}  // namespace

extern "C" {

void kllm_chip_close(kllm_chip *chip) {
    if (!chip) return;
    if (chip->ctx) tape_ctx_destroy(chip->ctx);
    for (auto &m : chip->maps) munmap(m.first, m.second);
    delete chip;
}

kllm_chip *kllm_chip_open(const char *dir_c) {
    if (!dir_c) {
        set_error("kllm_chip_open: NULL directory");
        return nullptr;
    }
    std::string dir(dir_c);
    kllm_chip *c = new kllm_chip();
    auto fail = [&]() -> kllm_chip * {
        kllm_chip_close(c);
        return nullptr;
    };
    std::vector<uint8_t> pj;
    if (!read_file(dir + "/processor.json", pj)) return fail();
    std::string js(pj.begin(), pj.end());
    c->vocab = json_int(js, "vocab_size");
    c->hidden = json_int(js, "hidden_dim");
    c->layers = json_int(js, "num_layers");
    c->n_kv = json_int(js, "num_kv_heads");
    c->head_dim = json_int(js, "head_dim");
    c->max_seq = json_int(js, "max_seq_len");
    c->eos = json_int(js, "eos_token_id");
    if (c->vocab <= 0 || c->hidden <= 0 || c->layers < 0 || c->n_kv <= 0 || c->head_dim <= 0 ||
        c->max_seq <= 0) {
        set_error("%s/processor.json: missing or invalid machine dimensions", dir_c);
        return fail();
    }
    c->embed_slot = json_nested(js, "input_map", "token_embed");
    c->cos_slot = json_nested(js, "input_map", "rope_cos");
    c->sin_slot = json_nested(js, "input_map", "rope_sin");
    c->logits_slot = json_nested(js, "output_map", "logits");
    c->kv_in.resize(2 * (size_t)c->layers);
    c->kv_out.resize(2 * (size_t)c->layers);
    for (int l = 0; l < c->layers; l++) {
        char k[64];
        snprintf(k, sizeof k, "L%d/cache_k", l);
        c->kv_in[2 * l] = json_nested(js, "input_map", k);
        snprintf(k, sizeof k, "L%d/cache_v", l);
        c->kv_in[2 * l + 1] = json_nested(js, "input_map", k);
        snprintf(k, sizeof k, "L%d/new_k", l);
        c->kv_out[2 * l] = json_nested(js, "output_map", k);
        snprintf(k, sizeof k, "L%d/new_v", l);
        c->kv_out[2 * l + 1] = json_nested(js, "output_map", k);
    }

    size_t V = c->vocab, H = c->hidden, S = c->max_seq, hd = c->head_dim;
    if (!read_array(dir + "/tables/embed_table.bin", c->embed, V * H)) return fail();
    if (!read_array(dir + "/tables/rope_cos.bin", c->rope_cos, S * hd)) return fail();
    if (!read_array(dir + "/tables/rope_sin.bin", c->rope_sin, S * hd)) return fail();

    std::string bpe = dir + "/bpe/";
    std::vector<uint8_t> meta;
    if (!read_file(bpe + "vocab_hash_keys.json", meta)) return fail();
    std::string ms(meta.begin(), meta.end());
    size_t sp = ms.find("shape");
    if (sp != std::string::npos && (sp = ms.find('[', sp)) != std::string::npos) {
        c->table_size = atoi(ms.c_str() + sp + 1);
        size_t cm = ms.find(',', sp);
        if (cm != std::string::npos) c->max_piece_len = atoi(ms.c_str() + cm + 1);
    }
    if (c->table_size < 0 || c->max_piece_len < 0) {
        set_error("%svocab_hash_keys.json: invalid shape", bpe.c_str());
        return fail();
    }
    size_t ts = c->table_size;
    if (!read_array(bpe + "vocab_hash_keys.bin", c->hash_keys, ts * c->max_piece_len) ||
        !read_array(bpe + "vocab_hash_vals.bin", c->hash_vals, ts) ||
        !read_array(bpe + "vocab_hash_lens.bin", c->hash_lens, ts) ||
        !read_array(bpe + "merge_a.bin", c->merge_a)) return fail();
    size_t nm = c->merge_a.size();
    if (!read_array(bpe + "merge_b.bin", c->merge_b, nm) ||
        !read_array(bpe + "merge_result.bin", c->merge_result, nm) ||
        !read_array(bpe + "special_ids.bin", c->special) ||
        !read_array(bpe + "id_to_bytes.bin", c->id_to_bytes) ||
        !read_array(bpe + "id_to_offsets.bin", c->id_to_offsets, V * 2)) return fail();
    c->bos = c->special.size() > 1 ? c->special[1] : 1;   // kllm.c:274-275
    for (size_t t = 0; t < V; t++) {
        long long off = c->id_to_offsets[2 * t], len = c->id_to_offsets[2 * t + 1];
        if (off < 0 || len < 0 || off + len > (long long)c->id_to_bytes.size()) {
            set_error("%sid_to_offsets.bin: entry %zu outside id_to_bytes", bpe.c_str(), t);
            return fail();
        }
    }

    std::string circ = dir + "/circuit/";
    std::vector<uint8_t> tape, slots;
    if (!read_file(circ + "tape.bin", tape) || !read_file(circ + "slots.bin", slots)) return fail();
    if (tape.size() < 8 || slots.size() < 4) {
        set_error("%s: truncated tape.bin / slots.bin", circ.c_str());
        return fail();
    }
    int32_t n_instr, isz, n_slots;
    memcpy(&n_instr, tape.data(), 4);
    memcpy(&isz, tape.data() + 4, 4);
    memcpy(&n_slots, slots.data(), 4);
    if (isz != (int)sizeof(TapeInstr)) {   // kllm.c:312-316
        set_error("tape instr size mismatch: file=%d, expected %zu", isz, sizeof(TapeInstr));
        return fail();
    }
    if (n_instr < 0 || n_slots < 0 || tape.size() != 8 + (size_t)n_instr * isz ||
        slots.size() != 4 + (size_t)n_slots * 40) {
        set_error("%s: tape.bin / slots.bin sizes disagree with their headers", circ.c_str());
        return fail();
    }
    auto slot_ok = [&](int s) { return s >= 0 && s < n_slots; };
    bool maps_ok = slot_ok(c->embed_slot) && slot_ok(c->cos_slot) && slot_ok(c->sin_slot) &&
                   slot_ok(c->logits_slot);
    for (int s : c->kv_in) maps_ok = maps_ok && slot_ok(s);
    for (int s : c->kv_out) maps_ok = maps_ok && slot_ok(s);
    if (!maps_ok) {
        set_error("%s/processor.json: slot map refers to a slot outside slots.bin", dir_c);
        return fail();
    }
    c->ctx = tape_ctx_create(n_slots, n_instr);
    if (n_instr) memcpy(c->ctx->tape, tape.data() + 8, (size_t)n_instr * isz);
    const uint8_t *rec = slots.data() + 4;
    for (int s = 0; s < n_slots; s++, rec += 40) {
        int32_t f[10];
        memcpy(f, rec, 40);
        int type = f[0], ndim = f[1];
        if (type == 0) continue;
        if (ndim < 0 || ndim > MAX_DIMS) {
            set_error("slots.bin: slot %d has ndim %d", s, ndim);
            return fail();
        }
        const int *shape = f + 2;
        char name[96];
        if (type == 4) {
            if (ndim != 2 || shape[0] < 0 || shape[1] < 0) {
                set_error("slots.bin: truth-table slot %d is not 2-D", s);
                return fail();
            }
            size_t K = shape[0], N = shape[1];
            std::vector<float> cb;
            snprintf(name, sizeof name, "const_%d_codebook.bin", s);
            if (!read_array(circ + name, cb)) return fail();
            if (cb.empty() || cb.size() > 65536) {
                set_error("slot %d: codebook of %zu entries", s, cb.size());
                return fail();
            }
            snprintf(name, sizeof name, "const_%d_indices.bin", s);
            uint16_t *ix = nullptr;
            if (K > 0 && N > 0) {   // mapped, not read: the upload copies it to HBM once
                ix = (uint16_t *)map_file(circ + name, K * N * 2, c->maps);
                if (!ix) return fail();
            } else {
                std::vector<uint16_t> e;
                if (!read_array(circ + name, e, 0)) return fail();
                c->ibufs.push_back(std::move(e));
                ix = c->ibufs.back().data();
            }
            c->fbufs.push_back(std::move(cb));
            tape_slot_set_truth_table(c->ctx, s, c->fbufs.back().data(),
                                      (int)c->fbufs.back().size(), ix, (int)K, (int)N);
        } else if (type == 1) {
            std::vector<float> d;
            snprintf(name, sizeof name, "const_%d.bin", s);
            if (!read_array(circ + name, d, (size_t)kllm::dims_size(shape, ndim))) return fail();
            c->fbufs.push_back(std::move(d));
            tape_slot_set_external(c->ctx, s, c->fbufs.back().data(), shape, ndim);
        } else {
            tape_slot_alloc(c->ctx, s, shape, ndim);
        }
    }
    return c;
}

TapeCtx *kllm_chip_ctx(kllm_chip *chip) { return chip ? chip->ctx : nullptr; }

int kllm_chip_info(kllm_chip *c, int *info) {
    if (!c || !info) return -1;
    int v[18] = {c->vocab, c->hidden, c->layers, c->n_kv, c->head_dim, c->max_seq, c->eos,
                 c->logits_slot, c->embed_slot, c->cos_slot, c->sin_slot, c->ctx->n_slots,
                 c->ctx->n_instrs, c->bos, c->table_size, c->max_piece_len,
                 (int)c->merge_a.size(), (int)c->special.size()};
    memcpy(info, v, sizeof v);
    return 0;
}

int kllm_chip_infer(kllm_chip *c, const int *prompt, int prompt_len, int max_new, int eos,
                    int *out, int *out_len) {
    if (!c) {
        set_error("kllm_chip_infer: NULL chip");
        return -1;
    }
    if (prompt_len + std::max(max_new, 0) > c->max_seq) {
        set_error("kllm_chip_infer: %d positions exceed the chip's RoPE table of %d",
                  prompt_len + max_new, c->max_seq);
        return -1;
    }
    return processor_infer(c->ctx, c->embed.data(), c->vocab, c->hidden, c->rope_cos.data(),
                           c->rope_sin.data(), c->head_dim, c->embed_slot, c->cos_slot,
                           c->sin_slot, c->kv_in.data(), c->kv_out.data(), c->logits_slot,
                           c->layers, c->n_kv, prompt, prompt_len, max_new, eos, out, out_len);
}

int kllm_chip_infer_batch(kllm_chip *c, const int *prompts, const int *prompt_lens, int nseq,
                          int max_new, int eos, int *out, int *out_lens) {
    if (!c || !prompt_lens || nseq < 1) {
        set_error("kllm_chip_infer_batch: bad argument");
        return -1;
    }
    for (int i = 0; i < nseq; i++)
        if (prompt_lens[i] + std::max(max_new, 0) > c->max_seq) {
            set_error("kllm_chip_infer_batch: sequence %d: %d positions exceed the chip's RoPE "
                      "table of %d", i, prompt_lens[i] + max_new, c->max_seq);
            return -1;
        }
    if (kllm_chip_plan_prepare(c) != 0) return -1;
    return kllm_infer_batch(c->ctx, prompts, prompt_lens, nseq, max_new, eos, out, out_lens);
}

int kllm_chip_plan_prepare(kllm_chip *c) {
    if (!c) {
        set_error("kllm_chip_plan_prepare: NULL chip");
        return -1;
    }
    return kllm_plan_prepare(c->ctx, c->embed.data(), c->vocab, c->hidden, c->rope_cos.data(),
                             c->rope_sin.data(), c->head_dim, c->embed_slot, c->cos_slot,
                             c->sin_slot, c->kv_in.data(), c->kv_out.data(), c->logits_slot,
                             c->layers, c->n_kv, c->max_seq);
}

int kllm_chip_infer_bytes(kllm_chip *c, const uint8_t *in, int len, int max_new, int max_seq,
                          token_callback_fn cb, void *ud, int *total) {
    if (!c) {
        set_error("kllm_chip_infer_bytes: NULL chip");
        return -1;
    }
    if (max_seq <= 0 || max_seq > c->max_seq) max_seq = c->max_seq;
    return processor_infer_bytes(
        c->ctx, c->hash_keys.data(), c->hash_vals.data(), c->hash_lens.data(), c->table_size,
        c->max_piece_len, c->merge_a.data(), c->merge_b.data(), c->merge_result.data(),
        (int)c->merge_a.size(), c->id_to_bytes.data(), c->id_to_offsets.data(),
        c->special.data(), (int)c->special.size(), c->bos, c->embed.data(), c->vocab, c->hidden,
        c->rope_cos.data(), c->rope_sin.data(), c->head_dim, c->embed_slot, c->cos_slot,
        c->sin_slot, c->kv_in.data(), c->kv_out.data(), c->logits_slot, c->layers, c->n_kv, in,
        len, max_new, c->eos, max_seq, 8192, cb, ud, total);
}

int kllm_chip_encode(kllm_chip *c, const uint8_t *bytes, int len, int max_tokens, int32_t *out) {
    if (!c || max_tokens < 1) return -1;
    return bpe_encode(bytes, len, c->hash_keys.data(), c->hash_vals.data(), c->hash_lens.data(),
                      c->table_size, c->max_piece_len, c->merge_a.data(), c->merge_b.data(),
                      c->merge_result.data(), (int)c->merge_a.size(), c->bos, max_tokens,
                      c->id_to_bytes.data(), c->id_to_offsets.data(), c->special.data(),
                      (int)c->special.size(), c->vocab, out);
}

int kllm_chip_decode(kllm_chip *c, const int32_t *ids, int n, int max_bytes, int skip,
                     uint8_t *out) {
    if (!c) return -1;
    return bpe_decode(ids, n, c->id_to_bytes.data(), c->id_to_offsets.data(), c->vocab,
                      c->special.data(), (int)c->special.size(), max_bytes, skip, out);
}

}  // extern "C"
