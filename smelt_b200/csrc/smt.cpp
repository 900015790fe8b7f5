// SMT container loader for the C-ABI (the reference's Engine::load, gpt2.rs:43-89, over
// PackReader, format.rs:94-175): the file is mapped read-only, the merkle content_id and the
// per-tensor BLAKE3 digests are verified (gpt2.rs:91-110), META gives the architecture and the
// TENSORS records become gpt2q_tensor_desc entries pointing into the mapping, which
// gpt2q_create uploads. Layout: 128-byte superheader (magic "SMT\x01", content_id at 16,
// file length at 48), then sections `type u32 | flags u32 | len u64 | payload`; TENSORS payload
// `[u32 count][u32 json_len][records JSON][tensor bytes]`.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "blake3.h"
#include "gpt2q.h"

namespace gpt2q {
void set_global_error(const std::string& msg);

namespace {

// ---- a small JSON reader: objects, arrays, strings, numbers, true/false/null ----
struct JVal {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    double num = 0;
    bool b = false;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal* get(const std::string& k) const {
        for (auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char* p;
    const char* end;
    bool ok = true;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool lit(const char* s) {
        const size_t n = std::strlen(s);
        if ((size_t)(end - p) < n || std::strncmp(p, s, n) != 0) return ok = false;
        p += n;
        return true;
    }
    std::string string() {
        std::string out;
        if (p >= end || *p != '"') {
            ok = false;
            return out;
        }
        ++p;
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\' && p < end) {
                const char e = *p++;
                switch (e) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        unsigned v = 0;
                        for (int i = 0; i < 4 && p < end; ++i, ++p) {
                            const char h = *p;
                            v = v * 16 + (unsigned)(h >= 'a' ? h - 'a' + 10 : h >= 'A' ? h - 'A' + 10 : h - '0');
                        }
                        if (v < 0x80) {
                            out += (char)v;
                        } else if (v < 0x800) {
                            out += (char)(0xC0 | (v >> 6));
                            out += (char)(0x80 | (v & 0x3F));
                        } else {
                            out += (char)(0xE0 | (v >> 12));
                            out += (char)(0x80 | ((v >> 6) & 0x3F));
                            out += (char)(0x80 | (v & 0x3F));
                        }
                        break;
                    }
                    default: out += e;
                }
            } else {
                out += c;
            }
        }
        if (p >= end) {
            ok = false;
            return out;
        }
        ++p;
        return out;
    }
    JVal value(int depth = 0) {
        JVal v;
        ws();
        if (p >= end || depth > 64) {
            ok = false;
            return v;
        }
        const char c = *p;
        if (c == '{') {
            v.kind = JVal::OBJ;
            ++p;
            ws();
            if (p < end && *p == '}') {
                ++p;
                return v;
            }
            while (ok) {
                ws();
                std::string k = string();
                ws();
                if (p >= end || *p != ':') {
                    ok = false;
                    break;
                }
                ++p;
                JVal x = value(depth + 1);
                v.obj.emplace_back(std::move(k), std::move(x));
                ws();
                if (p < end && *p == ',') {
                    ++p;
                    continue;
                }
                if (p < end && *p == '}') {
                    ++p;
                    break;
                }
                ok = false;
            }
        } else if (c == '[') {
            v.kind = JVal::ARR;
            ++p;
            ws();
            if (p < end && *p == ']') {
                ++p;
                return v;
            }
            while (ok) {
                v.arr.push_back(value(depth + 1));
                ws();
                if (p < end && *p == ',') {
                    ++p;
                    continue;
                }
                if (p < end && *p == ']') {
                    ++p;
                    break;
                }
                ok = false;
            }
        } else if (c == '"') {
            v.kind = JVal::STR;
            v.str = string();
        } else if (c == 't') {
            v.kind = JVal::BOOL;
            v.b = lit("true");
        } else if (c == 'f') {
            v.kind = JVal::BOOL;
            lit("false");
        } else if (c == 'n') {
            lit("null");
        } else {
            v.kind = JVal::NUM;
            char* e = nullptr;
            const std::string s(p, (size_t)std::min<ptrdiff_t>(end - p, 64));
            v.num = std::strtod(s.c_str(), &e);
            if (e == s.c_str()) ok = false;
            p += (e - s.c_str());
        }
        return v;
    }
};

bool parse_json(const uint8_t* b, size_t n, JVal& out) {
    JParser jp{reinterpret_cast<const char*>(b), reinterpret_cast<const char*>(b) + n};
    out = jp.value();
    return jp.ok;
}

uint32_t rd32(const uint8_t* p) { uint32_t v; std::memcpy(&v, p, 4); return v; }
uint64_t rd64(const uint8_t* p) { uint64_t v; std::memcpy(&v, p, 8); return v; }

int hw_threads() {
    const unsigned n = std::thread::hardware_concurrency();
    return n == 0 ? 1 : (int)std::min(n, 64u);
}

std::string hex(const uint8_t* d, size_t n) {
    static const char* H = "0123456789abcdef";
    std::string s;
    for (size_t i = 0; i < n; ++i) {
        s += H[d[i] >> 4];
        s += H[d[i] & 15];
    }
    return s;
}

struct Record {
    std::string name, atom;
    std::vector<int64_t> shape;
    uint64_t offset = 0, len = 0;
    std::string digest;  // 32 hex chars
    bool digest_ok = true;
};

struct Smt {
    const uint8_t* map = nullptr;
    size_t size = 0;
    int fd = -1;
    std::array<uint8_t, 32> content_id{};
    bool merkle_ok = false;
    gpt2q_config cfg{};
    std::vector<Record> recs;
    const uint8_t* tensors = nullptr;  // start of the tensor bytes
    std::string err;
    ~Smt() {
        if (map) munmap(const_cast<uint8_t*>(map), size);
        if (fd >= 0) close(fd);
    }
};

// Opens and parses `path`; with `verify`, checks the merkle content_id and every tensor digest.
bool open_smt(const char* path, bool verify, Smt& s) {
    s.fd = open(path, O_RDONLY);
    if (s.fd < 0) return s.err = std::string("cannot open ") + path, false;
    struct stat st;
    if (fstat(s.fd, &st) != 0 || st.st_size < 128) return s.err = "not an SMT container (too short)", false;
    s.size = (size_t)st.st_size;
    void* m = mmap(nullptr, s.size, PROT_READ, MAP_PRIVATE, s.fd, 0);
    if (m == MAP_FAILED) return s.err = "mmap failed", false;
    s.map = static_cast<const uint8_t*>(m);
    if (std::memcmp(s.map, "SMT\x01", 4) != 0) return s.err = "bad magic", false;
    std::memcpy(s.content_id.data(), s.map + 16, 32);
    // sections
    std::map<uint32_t, std::pair<size_t, size_t>> sec;  // type -> (payload offset, len)
    std::vector<std::array<uint8_t, 32>> digests;
    size_t off = 128;
    while (off < s.size) {
        if (off + 16 > s.size) return s.err = "truncated section header", false;
        const uint32_t ty = rd32(s.map + off);
        const uint64_t len = rd64(s.map + off + 8);
        const size_t p = off + 16;
        if (len > s.size - p) return s.err = "section runs past the end of the file", false;
        if (!sec.count(ty)) sec[ty] = {p, (size_t)len};
        if (verify) {
            std::array<uint8_t, 32> d;
            blake3(s.map + p, (size_t)len, d.data(), hw_threads());
            digests.push_back(d);
        }
        off = p + (size_t)len;
    }
    if (verify) {
        std::sort(digests.begin(), digests.end());
        std::array<uint8_t, 32> cid;
        blake3(digests.data(), digests.size() * 32, cid.data());
        s.merkle_ok = cid == s.content_id;
        if (!s.merkle_ok) return s.err = "merkle content_id mismatch", false;
    }
    // META
    if (!sec.count(2)) return s.err = "missing META section", false;
    JVal meta;
    if (!parse_json(s.map + sec[2].first, sec[2].second, meta)) return s.err = "META is not valid JSON", false;
    const JVal* arch = meta.get("arch");
    auto num = [&](const char* k, double& v) {
        const JVal* x = arch ? arch->get(k) : nullptr;
        if (!x || x->kind != JVal::NUM) return false;
        v = x->num;
        return true;
    };
    double ne, nl, nh, nc, vs, eps;
    if (!num("n_embd", ne) || !num("n_layer", nl) || !num("n_head", nh) || !num("n_ctx", nc) ||
        !num("vocab_size", vs) || !num("ln_eps", eps))
        return s.err = "META.arch lacks n_embd/n_layer/n_head/n_ctx/vocab_size/ln_eps", false;
    s.cfg.n_embd = (int32_t)ne;
    s.cfg.n_layer = (int32_t)nl;
    s.cfg.n_head = (int32_t)nh;
    s.cfg.n_ctx = (int32_t)nc;
    s.cfg.vocab = (int32_t)vs;
    s.cfg.ln_eps = (float)eps;
    // TENSORS
    if (!sec.count(5)) return s.err = "missing TENSORS section", false;
    const uint8_t* t = s.map + sec[5].first;
    const size_t tlen = sec[5].second;
    if (tlen < 8) return s.err = "TENSORS section too short", false;
    const uint32_t count = rd32(t), json_len = rd32(t + 4);
    if (8 + (size_t)json_len > tlen) return s.err = "TENSORS records run past the section", false;
    JVal recs;
    if (!parse_json(t + 8, json_len, recs) || recs.kind != JVal::ARR) return s.err = "TENSORS records are not a JSON array", false;
    if (recs.arr.size() != count) return s.err = "tensor count mismatch", false;
    s.tensors = t + 8 + json_len;
    const size_t avail = tlen - 8 - json_len;
    for (const JVal& r : recs.arr) {
        Record rec;
        const JVal *n = r.get("name"), *a = r.get("atom"), *sh = r.get("shape"), *o = r.get("offset"),
                   *l = r.get("len"), *d = r.get("digest");
        if (!n || !a || !sh || !o || !l || sh->kind != JVal::ARR || o->kind != JVal::NUM || l->kind != JVal::NUM ||
            o->num < 0 || l->num < 0 || o->num > 9.0e15 || l->num > 9.0e15)
            return s.err = "malformed tensor record", false;
        for (const JVal& x : sh->arr)
            if (x.kind != JVal::NUM || x.num < 0 || x.num > 2147483647.0) return s.err = "malformed tensor shape", false;
        rec.name = n->str;
        rec.atom = a->str;
        for (const JVal& x : sh->arr) rec.shape.push_back((int64_t)x.num);
        rec.offset = (uint64_t)o->num;
        rec.len = (uint64_t)l->num;
        rec.digest = d ? d->str : "";
        if (rec.offset > avail || rec.len > avail - rec.offset) return s.err = "tensor " + rec.name + " runs past the section", false;
        s.recs.push_back(std::move(rec));
    }
    if (verify) {  // per-tensor digests (verify_tensor_digests, gpt2.rs:91-110), tensors spread over threads
        std::atomic<size_t> next{0};
        auto work = [&] {
            for (size_t i; (i = next.fetch_add(1)) < s.recs.size();) {
                Record& r = s.recs[i];
                uint8_t h[32];
                blake3(s.tensors + r.offset, (size_t)r.len, h);
                r.digest_ok = hex(h, 16) == r.digest;
            }
        };
        std::vector<std::thread> pool;
        for (int t = 1; t < hw_threads(); ++t) pool.emplace_back(work);
        work();
        for (auto& t : pool) t.join();
        for (const Record& r : s.recs)
            if (!r.digest_ok) return s.err = "digest mismatch: " + r.name, false;
    }
    return true;
}

}  // namespace
}  // namespace gpt2q

using namespace gpt2q;

extern "C" {

int gpt2q_blake3(const void* data, uint64_t len, uint8_t* out32) {
    if ((!data && len) || !out32) return GPT2Q_EARG;
    blake3(data, (size_t)len, out32, hw_threads());
    return GPT2Q_OK;
}

int gpt2q_smt_inspect(const char* path, int verify, char* json, size_t cap) {
    if (!path || !json || cap == 0) return GPT2Q_EARG;
    Smt s;
    if (!open_smt(path, verify != 0, s)) {
        set_global_error("SMT: " + s.err);
        return GPT2Q_EARG;
    }
    std::string o = "{\"content_id\": \"" + hex(s.content_id.data(), 32) + "\", \"verified\": " +
                    (verify ? "true" : "false") + ", \"arch\": {\"n_embd\": " + std::to_string(s.cfg.n_embd) +
                    ", \"n_layer\": " + std::to_string(s.cfg.n_layer) + ", \"n_head\": " +
                    std::to_string(s.cfg.n_head) + ", \"n_ctx\": " + std::to_string(s.cfg.n_ctx) +
                    ", \"vocab_size\": " + std::to_string(s.cfg.vocab) + "}, \"tensors\": [";
    for (size_t i = 0; i < s.recs.size(); ++i) {
        const Record& r = s.recs[i];
        o += (i ? ", " : "") + std::string("{\"name\": \"") + r.name + "\", \"atom\": \"" + r.atom + "\", \"len\": " +
             std::to_string(r.len) + ", \"shape\": [";
        for (size_t k = 0; k < r.shape.size(); ++k) o += (k ? ", " : "") + std::to_string(r.shape[k]);
        o += "]}";
    }
    o += "]}";
    if (o.size() + 1 > cap) return GPT2Q_EARG;
    std::memcpy(json, o.c_str(), o.size() + 1);
    return GPT2Q_OK;
}

int gpt2q_create_from_smt(const char* path, int device, int max_seqs, int max_tokens, int verify,
                          gpt2q_handle** out) {
    if (!path || !out) return GPT2Q_EARG;
    *out = nullptr;
    Smt s;
    if (!open_smt(path, verify != 0, s)) {
        set_global_error("SMT: " + s.err);
        return GPT2Q_EARG;
    }
    gpt2q_config cfg = s.cfg;
    cfg.max_seqs = max_seqs;
    cfg.max_tokens = max_tokens;
    std::vector<gpt2q_tensor_desc> d(s.recs.size());
    for (size_t i = 0; i < s.recs.size(); ++i) {
        const Record& r = s.recs[i];
        if (r.shape.empty() || r.shape.size() > 2) {
            set_global_error("SMT: tensor " + r.name + " has rank other than 1 or 2");
            return GPT2Q_EARG;
        }
        d[i].name = r.name.c_str();
        d[i].atom = r.atom.c_str();
        d[i].ndim = (int32_t)r.shape.size();
        d[i].shape[0] = r.shape[0];
        d[i].shape[1] = r.shape.size() > 1 ? r.shape[1] : 0;
        d[i].data = s.tensors + r.offset;
        d[i].len = r.len;
    }
    // gpt2q_create copies every payload to the device before it returns
    return gpt2q_create(&cfg, d.data(), (int)d.size(), device, out);
}

}  // extern "C"
