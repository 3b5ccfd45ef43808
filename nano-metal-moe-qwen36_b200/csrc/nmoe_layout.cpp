// nmoe_layout.cpp -- layout.json validation (host only).
//
// The converter writes packed_experts*/layout.json with keys expert_size, num_layers,
// num_experts and components[{name, offset, size}] (scripts/convert_qwen36.py:351-359).
// The reference's validator (src/expert_io.m:274-316) is never called and would reject
// that file (it requires bits/dtype/shape keys the converter does not emit). This one
// accepts the converter's real output, and still checks dtype/shape/bits when present
// against the built-in layout (the rules of NMMBuildExpertLayout, src/expert_io.m:132-181).
#include <ctype.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "nmoe/moe_cuda.h"

namespace {

struct JVal {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    double num = 0;
    bool b = false;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal *get(const char *key) const {
        for (auto &kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char *p, *end;
    std::string err;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\t' || *p == '\r')) ++p;
    }
    bool fail(const char *m) {
        if (err.empty()) err = m;
        return false;
    }
    bool parse_string(std::string &out) {
        if (p >= end || *p != '"') return fail("expected string");
        ++p;
        while (p < end && *p != '"') {
            if (*p == '\\') {
                if (++p >= end) return fail("bad escape");
                switch (*p) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'u':
                        if (end - p < 5) return fail("bad \\u escape");
                        out += '?';
                        p += 4;
                        break;
                    default: out += *p;
                }
                ++p;
            } else {
                out += *p++;
            }
        }
        if (p >= end) return fail("unterminated string");
        ++p;
        return true;
    }
    bool parse(JVal &v, int depth = 0) {
        if (depth > 32) return fail("nesting too deep");
        ws();
        if (p >= end) return fail("unexpected end");
        if (*p == '{') {
            v.kind = JVal::Obj;
            ++p;
            ws();
            if (p < end && *p == '}') { ++p; return true; }
            for (;;) {
                ws();
                std::string k;
                if (!parse_string(k)) return false;
                ws();
                if (p >= end || *p != ':') return fail("expected ':'");
                ++p;
                JVal child;
                if (!parse(child, depth + 1)) return false;
                v.obj.emplace_back(k, std::move(child));
                ws();
                if (p < end && *p == ',') { ++p; continue; }
                if (p < end && *p == '}') { ++p; return true; }
                return fail("expected ',' or '}'");
            }
        }
        if (*p == '[') {
            v.kind = JVal::Arr;
            ++p;
            ws();
            if (p < end && *p == ']') { ++p; return true; }
            for (;;) {
                JVal child;
                if (!parse(child, depth + 1)) return false;
                v.arr.push_back(std::move(child));
                ws();
                if (p < end && *p == ',') { ++p; continue; }
                if (p < end && *p == ']') { ++p; return true; }
                return fail("expected ',' or ']'");
            }
        }
        if (*p == '"') { v.kind = JVal::Str; return parse_string(v.str); }
        if (!strncmp(p, "true", 4)) { v.kind = JVal::Bool; v.b = true; p += 4; return true; }
        if (!strncmp(p, "false", 5)) { v.kind = JVal::Bool; p += 5; return true; }
        if (!strncmp(p, "null", 4)) { v.kind = JVal::Null; p += 4; return true; }
        char *e = nullptr;
        std::string tmp(p, std::min<size_t>(64, end - p));
        double d = strtod(tmp.c_str(), &e);
        if (e == tmp.c_str()) return fail("bad value");
        v.kind = JVal::Num;
        v.num = d;
        p += (e - tmp.c_str());
        return true;
    }
};

struct Comp {
    const char *name;
    size_t rows, logical_cols, packed_cols;
    const char *dtype;
};

int set(char *err, size_t n, int code, const char *fmt, ...) {
    if (err && n) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err, n, fmt, ap);
        va_end(ap);
    }
    return code;
}

}  // namespace

extern "C" int nmoe_moe_validate_layout_json(const char *path, int quant_bits, char *err, size_t errlen) {
    if (err && errlen) err[0] = 0;
    if (path == nullptr || (quant_bits != 2 && quant_bits != 4))
        return set(err, errlen, NMOE_EINVAL, "bad path or quant_bits %d", quant_bits);
    FILE *f = fopen(path, "rb");
    if (!f) return set(err, errlen, NMOE_EIO, "cannot open %s", path);
    std::string text;
    char buf[4096];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) text.append(buf, n);
    fclose(f);
    JParser jp{text.data(), text.data() + text.size(), {}};
    JVal root;
    if (!jp.parse(root) || root.kind != JVal::Obj)
        return set(err, errlen, NMOE_ESIZE, "layout is not a JSON object: %s", jp.err.c_str());

    const size_t vpw = 32 / (size_t)quant_bits;
    const Comp comps[9] = {
        {"gate_proj.weight", NMOE_INTER, NMOE_HIDDEN, NMOE_HIDDEN / vpw, "u32"},
        {"gate_proj.scales", NMOE_INTER, NMOE_HIDDEN, NMOE_HIDDEN / NMOE_GROUP, "u16"},
        {"gate_proj.biases", NMOE_INTER, NMOE_HIDDEN, NMOE_HIDDEN / NMOE_GROUP, "u16"},
        {"up_proj.weight", NMOE_INTER, NMOE_HIDDEN, NMOE_HIDDEN / vpw, "u32"},
        {"up_proj.scales", NMOE_INTER, NMOE_HIDDEN, NMOE_HIDDEN / NMOE_GROUP, "u16"},
        {"up_proj.biases", NMOE_INTER, NMOE_HIDDEN, NMOE_HIDDEN / NMOE_GROUP, "u16"},
        {"down_proj.weight", NMOE_HIDDEN, NMOE_INTER, NMOE_INTER / vpw, "u32"},
        {"down_proj.scales", NMOE_HIDDEN, NMOE_INTER, NMOE_INTER / NMOE_GROUP, "u16"},
        {"down_proj.biases", NMOE_HIDDEN, NMOE_INTER, NMOE_INTER / NMOE_GROUP, "u16"},
    };
    size_t off[9];
    nmoe_moe_expert_offsets(quant_bits, off);
    const size_t esz = nmoe_moe_expert_size(quant_bits);

    if (const JVal *b = root.get("bits")) {
        if (b->kind != JVal::Num || (int)b->num != quant_bits)
            return set(err, errlen, NMOE_ESIZE, "bits key disagrees with quant_bits %d", quant_bits);
    }
    const JVal *es = root.get("expert_size");
    if (!es || es->kind != JVal::Num) return set(err, errlen, NMOE_ESIZE, "missing expert_size");
    if ((size_t)es->num != esz)
        return set(err, errlen, NMOE_ESIZE, "expert_size %lld does not match the q%d layout (%zu)", (long long)es->num, quant_bits, esz);
    for (const char *key : {"num_layers", "num_experts"}) {
        const JVal *v = root.get(key);
        if (v && (v->kind != JVal::Num || v->num < 1))
            return set(err, errlen, NMOE_ESIZE, "%s must be a positive number", key);
    }
    const JVal *cs = root.get("components");
    if (!cs || cs->kind != JVal::Arr || cs->arr.size() != 9)
        return set(err, errlen, NMOE_ESIZE, "components must be an array of 9 entries");
    for (int i = 0; i < 9; ++i) {
        const JVal &c = cs->arr[i];
        if (c.kind != JVal::Obj) return set(err, errlen, NMOE_ESIZE, "component %d is not an object", i);
        const JVal *name = c.get("name"), *o = c.get("offset"), *s = c.get("size");
        if (!name || name->kind != JVal::Str || !o || o->kind != JVal::Num || !s || s->kind != JVal::Num)
            return set(err, errlen, NMOE_ESIZE, "component %d lacks name/offset/size", i);
        if (name->str != comps[i].name)
            return set(err, errlen, NMOE_ESIZE, "unexpected component %s at index %d", name->str.c_str(), i);
        const size_t ebytes = (comps[i].dtype[1] == '3' ? 4 : 2) * comps[i].rows * comps[i].packed_cols;
        if ((size_t)o->num != off[i] || (size_t)s->num != ebytes)
            return set(err, errlen, NMOE_ESIZE, "component %s offset/size mismatch", comps[i].name);
        if (const JVal *dt = c.get("dtype")) {
            std::string d = dt->kind == JVal::Str ? dt->str : "";
            for (auto &ch : d) ch = (char)tolower(ch);
            if (d != comps[i].dtype)
                return set(err, errlen, NMOE_ESIZE, "component %s dtype mismatch", comps[i].name);
        }
        if (const JVal *sh = c.get("shape")) {
            if (sh->kind != JVal::Arr || sh->arr.size() != 2 || (size_t)sh->arr[0].num != comps[i].rows ||
                (size_t)sh->arr[1].num != comps[i].packed_cols)
                return set(err, errlen, NMOE_ESIZE, "component %s shape mismatch", comps[i].name);
        }
    }
    return NMOE_OK;
}
