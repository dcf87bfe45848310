// Checkpoint access for real GLM-5.3 weights: safetensors shards and the model.safetensors.index.json
// name -> shard map, read straight into host or device memory.
//
// Reference: the gx index (native/glm53/gx.vyb:1-120: gx_shard_for, gx_resolve: name -> shard from
// the index, then that shard's safetensors header for the byte range) over the safetensors reader
// (native/torchload/safetensors.vyb: u64 header length, JSON header {name: {dtype, shape,
// data_offsets}}, data region after it, offsets relative to it), and the shard sanity check of
// native/glm53/loader.py (a shard counts only if its header parses and the file holds the data
// region the header describes).  The index is parsed once per checkpoint; a shard's header once,
// when a name first resolves to it.
#include <sys/stat.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace vfmoe {

int read_range(FILE *f, int64_t off, int64_t n, char *dst, bool device, const char *what);

// ----------------------------------------------------------------------------- minimal JSON
// Objects, arrays, strings (\" \\ \/ \b \f \n \r \t \uXXXX), integers and the literals; enough for
// safetensors headers and the index (numbers there are integers).
struct Json {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    int64_t num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
    const Json *get(const char *key) const {
        for (auto &kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

struct JsonParser {
    const char *p, *end;
    bool ok = true;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    bool lit(const char *s) {
        const size_t n = strlen(s);
        if ((size_t)(end - p) < n || memcmp(p, s, n)) return ok = false;
        p += n;
        return true;
    }
    bool string(std::string &out) {
        if (p >= end || *p != '"') return ok = false;
        ++p;
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= end) return ok = false;
                c = *p++;
                switch (c) {
                    case '"': case '\\': case '/': out.push_back(c); break;
                    case 'b': out.push_back('\b'); break;
                    case 'f': out.push_back('\f'); break;
                    case 'n': out.push_back('\n'); break;
                    case 'r': out.push_back('\r'); break;
                    case 't': out.push_back('\t'); break;
                    case 'u': {
                        if (end - p < 4) return ok = false;
                        unsigned v = 0;
                        for (int i = 0; i < 4; ++i) {
                            const char h = *p++;
                            v = v * 16 + (h >= '0' && h <= '9' ? h - '0' : (h | 32) - 'a' + 10);
                        }
                        if (v < 0x80) {
                            out.push_back((char)v);
                        } else if (v < 0x800) {
                            out.push_back((char)(0xC0 | (v >> 6)));
                            out.push_back((char)(0x80 | (v & 63)));
                        } else {
                            out.push_back((char)(0xE0 | (v >> 12)));
                            out.push_back((char)(0x80 | ((v >> 6) & 63)));
                            out.push_back((char)(0x80 | (v & 63)));
                        }
                        break;
                    }
                    default: return ok = false;
                }
            } else {
                out.push_back(c);
            }
        }
        if (p >= end) return ok = false;
        ++p;
        return true;
    }
    bool value(Json &v, int depth = 0) {
        if (depth > 64) return ok = false;
        ws();
        if (p >= end) return ok = false;
        const char c = *p;
        if (c == '{') {
            v.kind = Json::OBJ;
            ++p;
            ws();
            if (p < end && *p == '}') {
                ++p;
                return true;
            }
            while (ok) {
                ws();
                std::string k;
                if (!string(k)) return false;
                ws();
                if (p >= end || *p != ':') return ok = false;
                ++p;
                v.obj.emplace_back(std::move(k), Json());
                if (!value(v.obj.back().second, depth + 1)) return false;
                ws();
                if (p < end && *p == ',') {
                    ++p;
                    continue;
                }
                if (p < end && *p == '}') {
                    ++p;
                    return true;
                }
                return ok = false;
            }
            return false;
        }
        if (c == '[') {
            v.kind = Json::ARR;
            ++p;
            ws();
            if (p < end && *p == ']') {
                ++p;
                return true;
            }
            while (ok) {
                v.arr.emplace_back();
                if (!value(v.arr.back(), depth + 1)) return false;
                ws();
                if (p < end && *p == ',') {
                    ++p;
                    continue;
                }
                if (p < end && *p == ']') {
                    ++p;
                    return true;
                }
                return ok = false;
            }
            return false;
        }
        if (c == '"') {
            v.kind = Json::STR;
            return string(v.str);
        }
        if (c == 't') {
            v.kind = Json::BOOL;
            v.num = 1;
            return lit("true");
        }
        if (c == 'f') {
            v.kind = Json::BOOL;
            return lit("false");
        }
        if (c == 'n') return lit("null");
        // number: integers; a fractional or exponent part is accepted and truncated
        v.kind = Json::NUM;
        bool neg = false;
        if (*p == '-') {
            neg = true;
            ++p;
        }
        if (p >= end || *p < '0' || *p > '9') return ok = false;
        int64_t n = 0;
        while (p < end && *p >= '0' && *p <= '9') n = n * 10 + (*p++ - '0');
        while (p < end && (*p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-' || (*p >= '0' && *p <= '9'))) ++p;
        v.num = neg ? -n : n;
        return true;
    }
};

static bool parse_json(const std::string &text, Json &out) {
    JsonParser jp{text.data(), text.data() + text.size()};
    return jp.value(out) && jp.ok;
}

// ----------------------------------------------------------------------------- checkpoint state
struct StTensor {
    int dtype = -1;
    std::vector<int64_t> shape;
    int64_t begin = 0, end = 0;  // absolute file offsets
};

struct Shard {
    std::string path;
    bool parsed = false;
    std::unordered_map<std::string, StTensor> tensors;
};

struct Checkpoint {
    std::string dir;
    std::vector<Shard> shards;
    std::unordered_map<std::string, int> shard_of;  // name -> shard (from the index)
    std::map<std::string, int> shard_index;          // file name -> shard
    std::mutex mu;
};

static std::mutex g_ck_mu;
static std::unordered_map<int64_t, std::unique_ptr<Checkpoint>> g_cks;
static int64_t g_next_ck = 1;

static int st_dtype(const std::string &s, int64_t *size) {
    static const struct {
        const char *name;
        int id, size;
    } t[] = {{"F32", VFMOE_ST_F32, 4},    {"F16", VFMOE_ST_F16, 2},     {"BF16", VFMOE_ST_BF16, 2},
             {"F64", VFMOE_ST_F64, 8},    {"I64", VFMOE_ST_I64, 8},     {"I32", VFMOE_ST_I32, 4},
             {"I16", VFMOE_ST_I16, 2},    {"I8", VFMOE_ST_I8, 1},       {"U8", VFMOE_ST_U8, 1},
             {"BOOL", VFMOE_ST_BOOL, 1},  {"U16", VFMOE_ST_U16, 2},     {"U32", VFMOE_ST_U32, 4},
             {"U64", VFMOE_ST_U64, 8},    {"F8_E4M3", VFMOE_ST_F8_E4M3, 1}, {"F8_E5M2", VFMOE_ST_F8_E5M2, 1}};
    for (auto &e : t)
        if (s == e.name) {
            *size = e.size;
            return e.id;
        }
    return -1;
}

static bool read_file(const std::string &path, std::string &out) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    char buf[1 << 16];
    size_t n;
    while ((n = fread(buf, 1, sizeof(buf), f)) > 0) out.append(buf, n);
    fclose(f);
    return true;
}

// Parse a shard's header (once): every tensor's dtype, shape and absolute byte range, checked
// against the header's own arithmetic and the file's size.
static int parse_shard(Shard &s) {
    if (s.parsed) return VFMOE_OK;
    FILE *f = fopen(s.path.c_str(), "rb");
    if (!f) {
        set_error("safetensors shard %s cannot be opened", s.path.c_str());
        return VFMOE_ERR_INVALID;
    }
    unsigned char lenb[8];
    int rc = VFMOE_OK;
    uint64_t hlen = 0;
    if (fread(lenb, 1, 8, f) != 8) rc = VFMOE_ERR_INVALID;
    for (int i = 0; i < 8; ++i) hlen |= (uint64_t)lenb[i] << (8 * i);
    struct stat stt;
    const int64_t fsize = stat(s.path.c_str(), &stt) == 0 ? (int64_t)stt.st_size : -1;
    if (!rc && (hlen == 0 || (int64_t)hlen > fsize - 8 || hlen > ((uint64_t)1 << 32))) rc = VFMOE_ERR_INVALID;
    std::string text;
    if (!rc) {
        text.resize(hlen);
        if (fread(&text[0], 1, hlen, f) != hlen) rc = VFMOE_ERR_INVALID;
    }
    fclose(f);
    Json h;
    if (!rc && (!parse_json(text, h) || h.kind != Json::OBJ)) rc = VFMOE_ERR_INVALID;
    if (rc) {
        set_error("safetensors shard %s: unreadable header", s.path.c_str());
        return rc;
    }
    const int64_t base = 8 + (int64_t)hlen;
    for (auto &kv : h.obj) {
        if (kv.first == "__metadata__") continue;
        const Json &t = kv.second;
        const Json *dt = t.get("dtype"), *sh = t.get("shape"), *off = t.get("data_offsets");
        int64_t esize = 0;
        StTensor st;
        if (!dt || dt->kind != Json::STR || !sh || sh->kind != Json::ARR || !off || off->kind != Json::ARR ||
            off->arr.size() != 2 || (st.dtype = st_dtype(dt->str, &esize)) < 0) {
            set_error("safetensors shard %s: malformed entry %s", s.path.c_str(), kv.first.c_str());
            return VFMOE_ERR_INVALID;
        }
        int64_t numel = 1;
        for (auto &d : sh->arr) {
            if (d.kind != Json::NUM || d.num < 0) {
                set_error("safetensors shard %s: bad shape of %s", s.path.c_str(), kv.first.c_str());
                return VFMOE_ERR_INVALID;
            }
            st.shape.push_back(d.num);
            numel *= d.num;
        }
        st.begin = base + off->arr[0].num;
        st.end = base + off->arr[1].num;
        if (off->arr[0].num < 0 || st.end < st.begin || st.end - st.begin != numel * esize || st.end > fsize) {
            set_error("safetensors shard %s: %s's byte range [%lld, %lld) is inconsistent or beyond the file "
                      "(%lld bytes)",
                      s.path.c_str(), kv.first.c_str(), (long long)st.begin, (long long)st.end, (long long)fsize);
            return VFMOE_ERR_INVALID;
        }
        s.tensors.emplace(kv.first, std::move(st));
    }
    s.parsed = true;
    return VFMOE_OK;
}

static int resolve(Checkpoint &ck, const char *name, Shard **sh, const StTensor **t) {
    std::lock_guard<std::mutex> lk(ck.mu);
    auto it = ck.shard_of.find(name);
    if (it == ck.shard_of.end()) {
        set_error("checkpoint %s: no tensor %s", ck.dir.c_str(), name);
        return VFMOE_ERR_INVALID;
    }
    Shard &s = ck.shards[it->second];
    if (int rc = parse_shard(s)) return rc;
    auto jt = s.tensors.find(name);
    if (jt == s.tensors.end()) {
        set_error("checkpoint %s: the index places %s in %s, whose header lacks it", ck.dir.c_str(), name,
                  s.path.c_str());
        return VFMOE_ERR_INVALID;
    }
    *sh = &s;
    *t = &jt->second;
    return VFMOE_OK;
}

static Checkpoint *get_ck(int64_t h) {
    std::lock_guard<std::mutex> lk(g_ck_mu);
    auto it = g_cks.find(h);
    if (it == g_cks.end()) {
        set_error("unknown checkpoint handle %lld", (long long)h);
        return nullptr;
    }
    return it->second.get();
}

}  // namespace vfmoe

using namespace vfmoe;

extern "C" {

int64_t vfmoe_ckpt_open(const char *dir) {
    if (!dir) {
        set_error("vfmoe_ckpt_open: null directory");
        return VFMOE_ERR_INVALID;
    }
    auto ck = std::make_unique<Checkpoint>();
    ck->dir = dir;
    std::string text;
    if (read_file(ck->dir + "/model.safetensors.index.json", text)) {
        Json idx;
        const Json *wm = nullptr;
        if (!parse_json(text, idx) || idx.kind != Json::OBJ || !(wm = idx.get("weight_map")) || wm->kind != Json::OBJ) {
            set_error("vfmoe_ckpt_open: %s/model.safetensors.index.json has no weight_map", dir);
            return VFMOE_ERR_INVALID;
        }
        for (auto &kv : wm->obj) {
            if (kv.second.kind != Json::STR || kv.second.str.find('/') != std::string::npos) {
                set_error("vfmoe_ckpt_open: bad shard name for %s", kv.first.c_str());
                return VFMOE_ERR_INVALID;
            }
            auto sit = ck->shard_index.find(kv.second.str);
            int si;
            if (sit == ck->shard_index.end()) {
                si = (int)ck->shards.size();
                ck->shards.emplace_back();
                ck->shards.back().path = ck->dir + "/" + kv.second.str;
                ck->shard_index.emplace(kv.second.str, si);
            } else {
                si = sit->second;
            }
            ck->shard_of.emplace(kv.first, si);
        }
    } else {
        // a single-file checkpoint: every tensor of model.safetensors
        ck->shards.emplace_back();
        ck->shards.back().path = ck->dir + "/model.safetensors";
        if (int rc = parse_shard(ck->shards.back())) return rc;
        for (auto &kv : ck->shards.back().tensors) ck->shard_of.emplace(kv.first, 0);
    }
    std::lock_guard<std::mutex> lk(g_ck_mu);
    const int64_t h = g_next_ck++;
    g_cks.emplace(h, std::move(ck));
    return h;
}

int vfmoe_ckpt_close(int64_t ck) {
    std::lock_guard<std::mutex> lk(g_ck_mu);
    if (!g_cks.erase(ck)) {
        set_error("unknown checkpoint handle %lld", (long long)ck);
        return VFMOE_ERR_HANDLE;
    }
    return VFMOE_OK;
}

int vfmoe_ckpt_find(int64_t ck, const char *name, vfmoe_tensor_info *info) {
    Checkpoint *c = get_ck(ck);
    if (!c) return VFMOE_ERR_HANDLE;
    if (!name || !info) {
        set_error("vfmoe_ckpt_find: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    Shard *s;
    const StTensor *t;
    if (int rc = resolve(*c, name, &s, &t)) return rc;
    memset(info, 0, sizeof(*info));
    info->dtype = t->dtype;
    info->ndim = (int64_t)t->shape.size();
    for (size_t i = 0; i < t->shape.size() && i < 8; ++i) info->shape[i] = t->shape[i];
    info->nbytes = t->end - t->begin;
    info->file_offset = t->begin;
    info->shard = (int64_t)(s - c->shards.data());
    if (t->shape.size() > 8) {
        set_error("vfmoe_ckpt_find: %s has %zu dimensions (8 supported)", name, t->shape.size());
        return VFMOE_ERR_UNSUPPORTED;
    }
    return VFMOE_OK;
}

int vfmoe_ckpt_read(int64_t ck, const char *name, int64_t dst, int64_t dst_bytes, int64_t device) {
    Checkpoint *c = get_ck(ck);
    if (!c) return VFMOE_ERR_HANDLE;
    if (!name || !dst) {
        set_error("vfmoe_ckpt_read: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    Shard *s;
    const StTensor *t;
    if (int rc = resolve(*c, name, &s, &t)) return rc;
    const int64_t n = t->end - t->begin;
    if (n > dst_bytes) {
        set_error("vfmoe_ckpt_read: %s is %lld bytes, the destination %lld", name, (long long)n, (long long)dst_bytes);
        return VFMOE_ERR_INVALID;
    }
    FILE *f = fopen(s->path.c_str(), "rb");
    if (!f) {
        set_error("vfmoe_ckpt_read: cannot open %s", s->path.c_str());
        return VFMOE_ERR_INVALID;
    }
    const int rc = read_range(f, t->begin, n, reinterpret_cast<char *>(dst), device != 0, name);
    fclose(f);
    return rc;
}

}  // extern "C"
