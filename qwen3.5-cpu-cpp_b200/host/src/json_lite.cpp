#include "json_lite.h"

#include <cstdlib>

namespace qwh {

namespace {
struct Parser {
    const char* p;
    const char* e;
    std::string err;
    int depth = 0;

    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool fail(const char* m) {
        if (err.empty()) err = m;
        return false;
    }
    bool lit(const char* s) {
        size_t n = 0;
        while (s[n]) ++n;
        if ((size_t)(e - p) < n) return false;
        for (size_t i = 0; i < n; ++i)
            if (p[i] != s[i]) return false;
        p += n;
        return true;
    }
    bool str(std::string& out) {
        if (p >= e || *p != '"') return fail("expected string");
        ++p;
        while (p < e && *p != '"') {
            if (*p == '\\') {
                if (++p >= e) return fail("bad escape");
                switch (*p) {
                    case 'n': out.push_back('\n'); break;
                    case 't': out.push_back('\t'); break;
                    case 'r': out.push_back('\r'); break;
                    case 'b': out.push_back('\b'); break;
                    case 'f': out.push_back('\f'); break;
                    case 'u': {
                        if (e - p < 5) return fail("bad \\u escape");
                        unsigned cp = (unsigned)std::strtoul(std::string(p + 1, p + 5).c_str(), nullptr, 16);
                        if (cp < 0x80) out.push_back((char)cp);
                        else if (cp < 0x800) { out.push_back((char)(0xC0 | (cp >> 6))); out.push_back((char)(0x80 | (cp & 0x3F))); }
                        else { out.push_back((char)(0xE0 | (cp >> 12))); out.push_back((char)(0x80 | ((cp >> 6) & 0x3F))); out.push_back((char)(0x80 | (cp & 0x3F))); }
                        p += 4;
                        break;
                    }
                    default: out.push_back(*p); break;
                }
                ++p;
            } else {
                out.push_back(*p++);
            }
        }
        if (p >= e) return fail("unterminated string");
        ++p;
        return true;
    }
    bool value(JValue& v) {
        if (++depth > 256) return fail("nesting too deep");
        ws();
        if (p >= e) return fail("unexpected end");
        bool ok = true;
        if (*p == '{') {
            v.kind = JValue::OBJ;
            ++p;
            ws();
            if (p < e && *p == '}') { ++p; --depth; return true; }
            while (true) {
                ws();
                std::string k;
                if (!str(k)) return false;
                ws();
                if (p >= e || *p != ':') return fail("expected ':'");
                ++p;
                v.obj.emplace_back(std::move(k), JValue());
                if (!value(v.obj.back().second)) return false;
                ws();
                if (p < e && *p == ',') { ++p; continue; }
                if (p < e && *p == '}') { ++p; break; }
                return fail("expected ',' or '}'");
            }
        } else if (*p == '[') {
            v.kind = JValue::ARR;
            ++p;
            ws();
            if (p < e && *p == ']') { ++p; --depth; return true; }
            while (true) {
                v.arr.emplace_back();
                if (!value(v.arr.back())) return false;
                ws();
                if (p < e && *p == ',') { ++p; continue; }
                if (p < e && *p == ']') { ++p; break; }
                return fail("expected ',' or ']'");
            }
        } else if (*p == '"') {
            v.kind = JValue::STR;
            ok = str(v.str);
        } else if (lit("true")) {
            v.kind = JValue::BOOL; v.b = true;
        } else if (lit("false")) {
            v.kind = JValue::BOOL; v.b = false;
        } else if (lit("null")) {
            v.kind = JValue::NUL;
        } else {
            const char* s = p;
            if (p < e && (*p == '-' || *p == '+')) ++p;
            while (p < e && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '-' || *p == '+')) ++p;
            if (p == s) return fail("unexpected character");
            v.kind = JValue::NUM;
            v.numtext.assign(s, p);
            char* endp = nullptr;
            v.num = std::strtod(v.numtext.c_str(), &endp);
            if (!endp || *endp) return fail("bad number");
        }
        --depth;
        return ok;
    }
};
}  // namespace

int64_t JValue::as_i64() const {
    if (kind != NUM) return 0;
    bool integral = numtext.find_first_of(".eE") == std::string::npos;
    return integral ? std::strtoll(numtext.c_str(), nullptr, 10) : (int64_t)num;
}

bool parse_json(const char* text, size_t n, JValue& out, std::string* err) {
    Parser ps{text, text + n, {}};
    bool ok = ps.value(out);
    if (ok) {
        ps.ws();
        if (ps.p != ps.e) ok = ps.fail("trailing characters");
    }
    if (!ok && err) *err = ps.err;
    return ok;
}

}  // namespace qwh
