// expert_store.cu — the fixed-Q4 expert layer store (FIXED_Q4_EXPERT_LAYER_V1,
// and the PBQ4EXPERT_LAYER_V1/V2 packs the reference upgrades to it) read
// into host or device memory as fixed-Q4 slot images: the HBM-resident
// expert table that replaces the reference's per-token pread streaming of
// expert slots.
//
// Store format (experts/mod.rs:44-50, :306-430, :2478-2484): a directory
// holding, per sparse layer N, layer_NN.json — serde JSON of
// ExpertLayerPackMetadata {format, layer, expert_size, experts, packs[{layer,
// expert, packed_bytes, records[{tensor, dtype, shape, source_offsets,
// source_hash?, record_offset, packed_bytes, groups, group_size,
// scale_bias_dtype}]}]} — and layer_NN.bin, expert e's slot at byte e *
// expert_size (expert_slot_offset, experts/store.rs:1154-1158). A fixed-Q4
// slot is the QwenMoeQ4ExpertLayout byte image (gate, up, down, each nibbles
// then bf16 scales then bf16 biases; model_family.rs:954-1010), one record
// per projection with record_offset at its nibbles, packed_bytes the nibble
// bytes and groups the scale count (fixed_q4_pack_from_pbq4_records,
// experts/slots.rs:984-1113).
//
// Validation restates ExpertLayerPackMetadata::validate (experts/mod.rs:
// 372-429) and checks each requested expert's records against the layout the
// caller expects. A PBQ4 slot holds a variable-length pack, parsed against
// its metadata and turned into the fixed image in memory, the conversion the
// reference applies when it rewrites such a layer (rewrite_pbq4_layer_to_
// fixed_q4, experts/mod.rs:2304-2375); files are never rewritten here. Host
// code only: the device upload is plain cudaMemcpyAsync of double-buffered
// pinned chunks of whole slots.

#include <algorithm>
#include <cctype>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <fcntl.h>
#include <unistd.h>

#include "kernels.h"

namespace {

// ---------------------------------------------------------------- minimal JSON
struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    bool integral = false;
    unsigned long long u = 0;  // when integral and non-negative
    double d = 0.0;
    std::string s;
    std::vector<Json> a;
    std::vector<std::pair<std::string, Json>> o;
    const Json* get(const char* key) const {
        for (const auto& kv : o)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

struct Parser {
    const char* p;
    const char* end;
    std::string err;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    bool fail(const char* what) {
        if (err.empty()) err = what;
        return false;
    }
    bool lit(const char* w) {
        const size_t n = std::strlen(w);
        if (size_t(end - p) < n || std::strncmp(p, w, n) != 0) return fail("bad literal");
        p += n;
        return true;
    }
    bool str(std::string& out) {
        if (p >= end || *p != '"') return fail("expected string");
        ++p;
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= end) return fail("bad escape");
                const char e = *p++;
                switch (e) {
                    case '"': case '\\': case '/': out += e; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'n': out += '\n'; break;
                    case 'r': out += '\r'; break;
                    case 't': out += '\t'; break;
                    case 'u': {  // names and dtypes are ASCII; keep the code unit as '?'
                        if (end - p < 4) return fail("bad \\u escape");
                        p += 4;
                        out += '?';
                        break;
                    }
                    default: return fail("bad escape");
                }
            } else {
                out += c;
            }
        }
        if (p >= end) return fail("unterminated string");
        ++p;
        return true;
    }
    bool num(Json& v) {
        const char* s = p;
        bool neg = false, frac = false;
        if (p < end && *p == '-') neg = true, ++p;
        while (p < end && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-')) {
            if (*p == '.' || *p == 'e' || *p == 'E') frac = true;
            ++p;
        }
        if (p == s) return fail("expected number");
        const std::string t(s, p);
        v.kind = Json::Number;
        v.d = std::strtod(t.c_str(), nullptr);
        if (!neg && !frac) {
            v.integral = true;
            v.u = std::strtoull(t.c_str(), nullptr, 10);
        }
        return true;
    }
    bool value(Json& v, int depth) {
        if (depth > 32) return fail("nesting too deep");
        ws();
        if (p >= end) return fail("unexpected end");
        const char c = *p;
        if (c == '{') {
            ++p;
            v.kind = Json::Object;
            ws();
            if (p < end && *p == '}') return ++p, true;
            for (;;) {
                ws();
                std::string k;
                if (!str(k)) return false;
                ws();
                if (p >= end || *p != ':') return fail("expected ':'");
                ++p;
                v.o.emplace_back(std::move(k), Json());
                if (!value(v.o.back().second, depth + 1)) return false;
                ws();
                if (p < end && *p == ',') { ++p; continue; }
                if (p < end && *p == '}') return ++p, true;
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            ++p;
            v.kind = Json::Array;
            ws();
            if (p < end && *p == ']') return ++p, true;
            for (;;) {
                v.a.emplace_back();
                if (!value(v.a.back(), depth + 1)) return false;
                ws();
                if (p < end && *p == ',') { ++p; continue; }
                if (p < end && *p == ']') return ++p, true;
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') return v.kind = Json::String, str(v.s);
        if (c == 't') return v.kind = Json::Bool, v.b = true, lit("true");
        if (c == 'f') return v.kind = Json::Bool, v.b = false, lit("false");
        if (c == 'n') return v.kind = Json::Null, lit("null");
        return num(v);
    }
};

struct Err {
    char* buf;
    size_t len;
    int fail(int code, const char* fmt, ...) {
        if (buf && len) {
            va_list ap;
            va_start(ap, fmt);
            vsnprintf(buf, len, fmt, ap);
            va_end(ap);
        }
        return code;
    }
};

bool get_u64(const Json& obj, const char* key, unsigned long long& out) {
    const Json* v = obj.get(key);
    if (!v || v->kind != Json::Number || !v->integral) return false;
    out = v->u;
    return true;
}

bool ends_with(const std::string& s, const char* suffix) {
    const size_t n = std::strlen(suffix);
    return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

std::string layer_file(const char* root, uint32_t layer, const char* ext) {
    char name[64];
    snprintf(name, sizeof name, "/layer_%02u.%s", layer, ext);
    return std::string(root) + name;
}

bool read_file(const std::string& path, std::string& out) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return false;
    char buf[1 << 16];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
    const bool ok = !std::ferror(f);
    std::fclose(f);
    return ok;
}

}  // namespace

// One record of a requested expert's pack metadata (ExpertPackRecord).
struct PackRec {
    std::string tensor;
    int proj = 0;  // 0 gate, 1 up, 2 down
    uint64_t record_offset = 0, packed_bytes = 0, groups = 0;
    bool bf16_scales = true;
};
// What the metadata says about the requested experts.
struct StoreInfo {
    bool fixed = true;            // a fixed image per slot (FIXED_Q4 / FIXED_MXFP4) or PBQ4 V1/V2 (pack per slot)
    bool mxfp4 = false;           // FIXED_MXFP4: records not checked (pack-level metadata only)
    uint64_t expert_size = 0;     // slot stride in layer_NN.bin
    std::vector<uint64_t> pack_bytes;        // per requested expert
    std::vector<std::vector<PackRec>> recs;  // per requested expert, in metadata order
};

static bool scale_dtype(const Json* sb, bool fixed, bool& bf16) {
    // serde default F32 (default_expert_scale_bias_dtype, experts/mod.rs:936-938)
    std::string d = sb ? (sb->kind == Json::String ? sb->s : std::string("?")) : std::string("F32");
    for (char& c : d) c = static_cast<char>(std::toupper(static_cast<unsigned char>(c)));
    if (d == "BF16" || d == "BFLOAT16") return bf16 = true, true;
    if (!fixed && (d == "F32" || d == "FLOAT32" || d == "FP32")) return bf16 = false, true;
    return false;
}

// Parse and validate layer `layer`'s metadata for the slots of experts
// [begin, begin + count) in layout L.
static int check_metadata(const char* root, uint32_t layer, const pbmoe_expert_layout* L, uint32_t begin,
                          uint32_t count, Err& e, StoreInfo& info) {
    const std::string path = layer_file(root, layer, "json");
    std::string text;
    if (!read_file(path, text))
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s cannot be read", path.c_str());
    Json meta;
    Parser ps{text.data(), text.data() + text.size(), {}};
    if (!ps.value(meta, 0) || meta.kind != Json::Object)
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "failed to parse expert metadata %s: %s", path.c_str(),
                      ps.err.empty() ? "not an object" : ps.err.c_str());
    const Json* fmt = meta.get("format");
    if (!fmt || fmt->kind != Json::String)
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s has no format", path.c_str());
    const bool mx_layout = L->encoding == PBMOE_EXPERT_MXFP4;
    if (mx_layout != (fmt->s == "FIXED_MXFP4_EXPERT_LAYER_V1"))
        return e.fail(PBMOE_ERR_UNSUPPORTED,
                      mx_layout ? "FlashMoe unsupported expert layout for %s: an MXFP4 layout reads only "
                                  "FIXED_MXFP4_EXPERT_LAYER_V1 layers, not %s"
                                : "FlashMoe unsupported expert layout for %s: format %s needs the fixed MXFP4 layout "
                                  "(encoding PBMOE_EXPERT_MXFP4)",
                      path.c_str(), fmt->s.c_str());
    if (fmt->s == "FIXED_Q4_EXPERT_LAYER_V1") {
        info.fixed = true;
    } else if (fmt->s == "FIXED_MXFP4_EXPERT_LAYER_V1") {
        info.fixed = info.mxfp4 = true;
        // the slot image of QwenMoeQ4ExpertLayout::fixed_mxfp4 (model_family.rs:846-952) for the layout's
        // shape: any other offsets would read the slot's bytes in the wrong places
        pbmoe_expert_layout want{};
        bool same = pbmoe_fixed_mxfp4_layout(L->hidden, L->intermediate, L->group_size, &want) == PBMOE_OK &&
                    want.expert_bytes == L->expert_bytes;
        for (int i = 0; same && i < 9; ++i) same = want.component_offsets[i] == L->component_offsets[i];
        if (!same)
            return e.fail(PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported expert layout for %s: an MXFP4 layer needs "
                          "the fixed MXFP4 layout of hidden %u, intermediate %u, group %u (E2M1 nibbles and E8M0 "
                          "scales per projection, no bias components)",
                          path.c_str(), L->hidden, L->intermediate, L->group_size);
    } else if (fmt->s == "PBQ4EXPERT_LAYER_V1" || fmt->s == "PBQ4EXPERT_LAYER_V2") {
        info.fixed = false;
    } else {
        return e.fail(PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported expert storage format %s in %s (this loader "
                      "reads FIXED_Q4_EXPERT_LAYER_V1, FIXED_MXFP4_EXPERT_LAYER_V1 and PBQ4EXPERT_LAYER_V1/V2)",
                      fmt->s.c_str(), path.c_str());
    }
    unsigned long long mlayer, expert_size, experts;
    if (!get_u64(meta, "layer", mlayer) || !get_u64(meta, "expert_size", expert_size) ||
        !get_u64(meta, "experts", experts))
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s lacks layer/expert_size/experts", path.c_str());
    if (mlayer != layer)
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s describes layer %llu, expected layer %u",
                      path.c_str(), mlayer, layer);
    if (expert_size == 0) return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s has zero expert_size", path.c_str());
    if (experts == 0) return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s has zero experts", path.c_str());
    if (info.fixed && expert_size != L->expert_bytes)
        return e.fail(PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported expert slot size %llu in %s (layout %llu bytes)",
                      expert_size, path.c_str(), static_cast<unsigned long long>(L->expert_bytes));
    if (uint64_t(begin) + count > experts)
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "experts [%u, %u) outside the %llu of %s", begin, begin + count,
                      experts, path.c_str());
    info.expert_size = expert_size;
    info.pack_bytes.assign(count, 0);
    info.recs.assign(count, {});
    const Json* packs = meta.get("packs");
    if (!packs || packs->kind != Json::Array)
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s has no packs", path.c_str());
    std::vector<char> seen(experts, 0);
    const uint64_t H = L->hidden, I = L->intermediate, G = L->group_size;
    const uint64_t shapes[3][2] = {{I, H}, {I, H}, {H, I}};
    const char* names[3] = {"gate_proj.weight", "up_proj.weight", "down_proj.weight"};
    for (const Json& pk : packs->a) {
        unsigned long long pl, ex, pb;
        if (pk.kind != Json::Object || !get_u64(pk, "layer", pl) || !get_u64(pk, "expert", ex))
            return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s has a malformed pack", path.c_str());
        if (pl != layer)
            return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s describes layer %llu expert %llu, expected "
                          "layer %u expert %llu", path.c_str(), pl, ex, layer, ex);
        if (ex >= experts)
            return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s describes expert %llu outside 0..%llu",
                          path.c_str(), ex, experts);
        if (seen[ex]) return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s has duplicate expert %llu", path.c_str(), ex);
        seen[ex] = 1;
        if (!get_u64(pk, "packed_bytes", pb)) pb = 0;  // serde default
        if (pb > expert_size)
            return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert metadata %s expert %llu length %llu exceeds slot size %llu",
                          path.c_str(), ex, pb, expert_size);
        if (ex < begin || ex >= uint64_t(begin) + count) continue;
        info.pack_bytes[ex - begin] = pb;
        if (info.mxfp4) continue;  // slot used as stored
        // the records of a requested expert must describe this layout: one
        // record per projection (in gate, up, down order for the fixed
        // image; found by suffix for a PBQ4 pack, pbq4_record_by_suffix)
        const Json* recs = pk.get("records");
        if (!recs || recs->kind != Json::Array || recs->a.size() != 3)
            return e.fail(PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported %s expert %llu in %s: expected gate, up "
                          "and down records", info.fixed ? "fixed-Q4" : "PBQ4", ex, path.c_str());
        std::vector<PackRec>& out = info.recs[ex - begin];
        info.pack_bytes[ex - begin] = pb;
        bool have[3] = {false, false, false};
        for (int q = 0; q < 3; ++q) {  // metadata order, which is the pack's record order
            const Json& r = recs->a[q];
            const Json* tn = r.get("tensor");
            int j = -1;
            for (int c = 0; c < 3 && tn && tn->kind == Json::String; ++c)
                if (ends_with(tn->s, names[c])) j = c;
            if (info.fixed && j != q) j = -1;  // the fixed image lists gate, up, down
            if (j < 0 || have[j])
                return e.fail(PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported %s expert %llu in %s: record %d is not a "
                              "%s record", info.fixed ? "fixed-Q4" : "PBQ4", ex, path.c_str(), q,
                              j < 0 ? names[q] : "distinct projection");
            have[j] = true;
            const Json* sh = r.get("shape");
            unsigned long long off, bytes, groups, gs;
            const bool ok = r.kind == Json::Object && get_u64(r, "record_offset", off) &&
                            get_u64(r, "packed_bytes", bytes) && get_u64(r, "groups", groups) &&
                            get_u64(r, "group_size", gs) && sh && sh->kind == Json::Array && sh->a.size() == 2 &&
                            sh->a[0].integral && sh->a[1].integral;
            if (!ok)
                return e.fail(PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported %s expert %llu in %s: record %d is not a "
                              "%s record", info.fixed ? "fixed-Q4" : "PBQ4", ex, path.c_str(), q, names[j]);
            const uint64_t rows = shapes[j][0], cols = shapes[j][1];
            bool bf16 = true;
            const bool match = sh->a[0].u == rows && sh->a[1].u == cols && gs == G && bytes == rows * cols / 2 &&
                               groups == rows * (cols / G) && scale_dtype(r.get("scale_bias_dtype"), info.fixed, bf16) &&
                               (!info.fixed || off == L->component_offsets[3 * j]);
            if (!match)
                return e.fail(PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported %s expert %llu in %s: %s does not "
                              "match the layout (hidden %llu, intermediate %llu, group %llu)",
                              info.fixed ? "fixed-Q4" : "PBQ4", ex, path.c_str(), tn->s.c_str(),
                              (unsigned long long)H, (unsigned long long)I, (unsigned long long)G);
            PackRec pr;
            pr.tensor = tn->s;
            pr.proj = j;
            pr.record_offset = off;
            pr.packed_bytes = bytes;
            pr.groups = groups;
            pr.bf16_scales = bf16;
            out.push_back(pr);
        }
    }
    for (uint64_t x = begin; x < uint64_t(begin) + count; ++x)
        if (!seen[x])
            return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert layer %u has no metadata for expert %llu", layer,
                          static_cast<unsigned long long>(x));
    return PBMOE_OK;
}

// pread of `bytes` at `offset`, all or nothing
static bool pread_all(int fd, void* dst, size_t bytes, uint64_t offset) {
    char* p = static_cast<char*>(dst);
    while (bytes) {
        const ssize_t n = pread(fd, p, bytes, static_cast<off_t>(offset));
        if (n <= 0) return false;
        p += n;
        bytes -= size_t(n);
        offset += uint64_t(n);
    }
    return true;
}
static uint16_t f32_to_bf16_rne(float v) {  // experts/slots.rs:1165-1169 (wrapping add)
    uint32_t bits;
    std::memcpy(&bits, &v, 4);
    const uint32_t lsb = (bits >> 16) & 1u;
    return static_cast<uint16_t>((bits + 0x7fffu + lsb) >> 16);
}

// One PBQ4 pack (PBQ4EXPERT magic, then per record: u32 name length, name,
// u64 nibble bytes, u64 groups, scales, biases, nibbles) parsed against its
// metadata as parse_pbq4_expert_pack_with_metadata (experts/mod.rs:546-653)
// does, and written as the fixed-Q4 slot image (fixed_q4_pack_from_pbq4_records,
// experts/slots.rs:984-1113; f32 scales/biases rounded to bf16).
static int assemble_pbq4(const uint8_t* pack, size_t len, const std::vector<PackRec>& recs,
                         const pbmoe_expert_layout* L, uint8_t* slot, uint32_t layer, uint64_t expert, Err& e) {
    static const char kMagic[] = "PBQ4EXPERT ";
    const size_t mlen = sizeof(kMagic) - 1;
    if (len < mlen || std::memcmp(pack, kMagic, mlen) != 0)
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "layer %u expert %llu: expert pack is missing PBQ4EXPERT header",
                      layer, (unsigned long long)expert);
    size_t cur = mlen;
    auto take = [&](size_t n) { const bool ok = n <= len - cur; return ok; };
    for (const PackRec& r : recs) {
        if (cur != r.record_offset)
            return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "layer %u expert %llu: tensor %s metadata offset mismatch: file "
                          "cursor %zu, metadata has %llu", layer, (unsigned long long)expert, r.tensor.c_str(), cur,
                          (unsigned long long)r.record_offset);
        uint32_t name_len;
        uint64_t packed_len, groups;
        if (!take(4)) goto short_pack;
        std::memcpy(&name_len, pack + cur, 4);
        cur += 4;
        if (!take(name_len)) goto short_pack;
        if (name_len != r.tensor.size() || std::memcmp(pack + cur, r.tensor.data(), name_len) != 0)
            return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "layer %u expert %llu: tensor name mismatch with metadata %s",
                          layer, (unsigned long long)expert, r.tensor.c_str());
        cur += name_len;
        if (!take(16)) goto short_pack;
        std::memcpy(&packed_len, pack + cur, 8);
        std::memcpy(&groups, pack + cur + 8, 8);
        cur += 16;
        if (packed_len != r.packed_bytes || groups != r.groups)
            return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "layer %u expert %llu: tensor %s length or group count differs "
                          "from its metadata", layer, (unsigned long long)expert, r.tensor.c_str());
        {
            const size_t eb = r.bf16_scales ? 2 : 4;
            if (!take(2 * groups * eb + packed_len)) goto short_pack;
            const uint8_t* sc = pack + cur;
            const uint8_t* bi = sc + groups * eb;
            const uint8_t* nib = bi + groups * eb;
            uint8_t* dw = slot + L->component_offsets[3 * r.proj];
            uint8_t* ds = slot + L->component_offsets[3 * r.proj + 1];
            uint8_t* db = slot + L->component_offsets[3 * r.proj + 2];
            std::memcpy(dw, nib, packed_len);
            if (r.bf16_scales) {
                std::memcpy(ds, sc, groups * 2);
                std::memcpy(db, bi, groups * 2);
            } else {
                for (uint64_t g = 0; g < groups; ++g) {
                    float f;
                    std::memcpy(&f, sc + 4 * g, 4);
                    const uint16_t hs = f32_to_bf16_rne(f);
                    std::memcpy(&f, bi + 4 * g, 4);
                    const uint16_t hb = f32_to_bf16_rne(f);
                    std::memcpy(ds + 2 * g, &hs, 2);
                    std::memcpy(db + 2 * g, &hb, 2);
                }
            }
            cur += 2 * groups * eb + packed_len;
        }
    }
    if (cur != len)
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "layer %u expert %llu: expert pack has %zu trailing bytes after "
                      "metadata records", layer, (unsigned long long)expert, len - cur);
    return PBMOE_OK;
short_pack:
    return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "layer %u expert %llu: expert pack is shorter than its records",
                  layer, (unsigned long long)expert);
}

static int open_slots(const char* root, uint32_t layer, const pbmoe_expert_layout* L, uint32_t begin,
                      uint32_t count, size_t dst_bytes, Err& e, int* fd_out, StoreInfo& info) {
    if (!root || !L || L->expert_bytes == 0)
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert layer read: null root or layout");
    if (count == 0) return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert layer read: no experts requested");
    if (dst_bytes < uint64_t(count) * L->expert_bytes)
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert layer read: %u slots of %llu bytes exceed the destination "
                      "(%zu bytes)", count, static_cast<unsigned long long>(L->expert_bytes), dst_bytes);
    const int rc = check_metadata(root, layer, L, begin, count, e, info);
    if (rc != PBMOE_OK) return rc;
    const std::string bin = layer_file(root, layer, "bin");
    const int fd = open(bin.c_str(), O_RDONLY);
    if (fd < 0) return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert layer %s cannot be opened", bin.c_str());
    const off_t size = lseek(fd, 0, SEEK_END);
    uint64_t need = (uint64_t(begin) + count) * info.expert_size;
    if (!info.fixed)
        need = uint64_t(begin + count - 1) * info.expert_size + info.pack_bytes[count - 1];
    if (size < 0 || uint64_t(size) < need) {
        close(fd);
        return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert layer %s is %lld bytes, shorter than experts [%u, %u)",
                      bin.c_str(), static_cast<long long>(size), begin, begin + count);
    }
    *fd_out = fd;
    return PBMOE_OK;
}

// Slots of requested experts [first, first + n) (relative to begin) into dst
// as fixed-Q4 images.
static int fill_slots(int fd, const StoreInfo& info, const pbmoe_expert_layout* L, uint32_t layer, uint32_t begin,
                      uint32_t first, uint32_t n, uint8_t* dst, Err& e) {
    if (info.fixed) {
        if (!pread_all(fd, dst, size_t(n) * L->expert_bytes, uint64_t(begin + first) * info.expert_size))
            return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert layer %u: read of experts [%u, %u) failed", layer,
                          begin + first, begin + first + n);
        return PBMOE_OK;
    }
    std::vector<uint8_t> pack;
    for (uint32_t k = 0; k < n; ++k) {
        const uint32_t x = first + k;
        pack.resize(info.pack_bytes[x]);
        if (!pread_all(fd, pack.data(), pack.size(), uint64_t(begin + x) * info.expert_size))
            return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert layer %u: read of expert %u failed", layer, begin + x);
        uint8_t* slot = dst + size_t(k) * L->expert_bytes;
        std::memset(slot, 0, L->expert_bytes);
        const int rc = assemble_pbq4(pack.data(), pack.size(), info.recs[x], L, slot, layer, begin + x, e);
        if (rc != PBMOE_OK) return rc;
    }
    return PBMOE_OK;
}

extern "C" int pbmoe_expert_layer_read(const char* root, uint32_t layer, const pbmoe_expert_layout* layout,
                                       uint32_t expert_begin, uint32_t expert_count, void* host_dst,
                                       size_t dst_bytes, char* error_buf, size_t error_len) {
    Err e{error_buf, error_len};
    if (!host_dst) return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert layer read: null destination");
    int fd = -1;
    StoreInfo info;
    int rc = open_slots(root, layer, layout, expert_begin, expert_count, dst_bytes, e, &fd, info);
    if (rc != PBMOE_OK) return rc;
    rc = fill_slots(fd, info, layout, layer, expert_begin, 0, expert_count, static_cast<uint8_t*>(host_dst), e);
    close(fd);
    return rc;
}

// Device upload through two pinned staging buffers of whole slots: while
// one chunk copies to the device, the next is read (and, for PBQ4 packs,
// assembled) from the file.
int pbmoe::expert_layer_upload(const char* root, uint32_t layer, const pbmoe_expert_layout* layout,
                               uint32_t expert_begin, uint32_t expert_count, void* device_dst, size_t dst_bytes,
                               cudaStream_t stream, char* error_buf, size_t error_len) {
    Err e{error_buf, error_len};
    if (!device_dst) return e.fail(PBMOE_ERR_INVALID_ARGUMENT, "expert layer load: null destination");
    int fd = -1;
    StoreInfo info;
    int rc = open_slots(root, layer, layout, expert_begin, expert_count, dst_bytes, e, &fd, info);
    if (rc != PBMOE_OK) return rc;
    const size_t slot = layout->expert_bytes;
    const uint32_t per_chunk = static_cast<uint32_t>(std::max<size_t>(1, (size_t(64) << 20) / slot));
    const size_t stage_bytes = size_t(per_chunk) * slot;
    void* stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    for (int i = 0; i < 2 && rc == PBMOE_OK; ++i) {
        if (cudaMallocHost(&stage[i], stage_bytes) != cudaSuccess ||
            cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) != cudaSuccess)
            rc = e.fail(PBMOE_ERR_CUDA, "expert layer load: pinned staging allocation failed");
    }
    for (uint32_t first = 0, i = 0; rc == PBMOE_OK && first < expert_count; first += per_chunk, ++i) {
        const int b = int(i & 1);
        const uint32_t n = std::min(per_chunk, expert_count - first);
        if (i >= 2 && cudaEventSynchronize(done[b]) != cudaSuccess) {
            rc = e.fail(PBMOE_ERR_CUDA, "expert layer load: staging wait failed");
            break;
        }
        rc = fill_slots(fd, info, layout, layer, expert_begin, first, n, static_cast<uint8_t*>(stage[b]), e);
        if (rc != PBMOE_OK) break;
        if (cudaMemcpyAsync(static_cast<char*>(device_dst) + size_t(first) * slot, stage[b], size_t(n) * slot,
                            cudaMemcpyHostToDevice, stream) != cudaSuccess ||
            cudaEventRecord(done[b], stream) != cudaSuccess)
            rc = e.fail(PBMOE_ERR_CUDA, "expert layer load: copy to the device failed");
    }
    for (int i = 0; i < 2; ++i) {
        if (done[i]) {
            cudaEventSynchronize(done[i]);
            cudaEventDestroy(done[i]);
        }
        if (stage[i]) cudaFreeHost(stage[i]);
    }
    close(fd);
    return rc;
}
