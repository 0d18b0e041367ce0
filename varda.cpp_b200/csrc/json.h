// Minimal JSON reader for the safetensors header and the model config (RFC 8259 subset: objects,
// arrays, strings with escapes, numbers, true/false/null). Objects keep their keys in a std::map;
// the config and header readers only look keys up, so key order does not matter.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"

namespace vb::json {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0;
    int64_t inum = 0;       // exact value for integer literals
    bool is_int = false;
    std::string str;
    std::vector<Value> arr;
    std::map<std::string, Value> obj;

    bool has(const std::string& k) const { return kind == Object && obj.count(k) != 0; }
    const Value& at(const std::string& k) const {
        if (kind != Object) fail(kFormat, "json: '" + k + "' looked up in a non-object");
        auto it = obj.find(k);
        if (it == obj.end()) fail(kFormat, "json: missing key '" + k + "'");
        return it->second;
    }
    const Value& at(size_t i) const {
        if (kind != Array || i >= arr.size()) fail(kFormat, "json: bad array index");
        return arr[i];
    }
    size_t size() const { return kind == Array ? arr.size() : kind == Object ? obj.size() : 0; }
    int64_t as_int(const char* what = "value") const {
        if (kind != Number) fail(kFormat, std::string("json: ") + what + " is not a number");
        if (is_int) return inum;
        if (num != static_cast<double>(static_cast<int64_t>(num))) fail(kFormat, std::string("json: ") + what + " is not an integer");
        return static_cast<int64_t>(num);
    }
    double as_num(const char* what = "value") const {
        if (kind != Number) fail(kFormat, std::string("json: ") + what + " is not a number");
        return is_int ? static_cast<double>(inum) : num;
    }
    const std::string& as_str(const char* what = "value") const {
        if (kind != String) fail(kFormat, std::string("json: ") + what + " is not a string");
        return str;
    }
    bool as_bool(const char* what = "value") const {
        if (kind != Bool) fail(kFormat, std::string("json: ") + what + " is not a boolean");
        return b;
    }
    std::vector<int> int_list(const char* what = "list") const {
        if (kind != Array) fail(kFormat, std::string("json: ") + what + " is not an array");
        std::vector<int> v;
        for (const auto& e : arr) v.push_back(static_cast<int>(e.as_int(what)));
        return v;
    }
    std::vector<int64_t> int64_list(const char* what = "list") const {
        if (kind != Array) fail(kFormat, std::string("json: ") + what + " is not an array");
        std::vector<int64_t> v;
        for (const auto& e : arr) v.push_back(e.as_int(what));
        return v;
    }
    std::vector<std::string> str_list(const char* what = "list") const {
        if (kind != Array) fail(kFormat, std::string("json: ") + what + " is not an array");
        std::vector<std::string> v;
        for (const auto& e : arr) v.push_back(e.as_str(what));
        return v;
    }
};

class Parser {
public:
    Parser(const char* b, const char* e) : p_(b), e_(e) {}
    Value parse_document() {
        Value v = value();
        ws();
        if (p_ != e_) err("trailing characters");
        return v;
    }

private:
    const char* p_;
    const char* e_;
    int depth_ = 0;

    [[noreturn]] void err(const char* m) { fail(kFormat, std::string("json: ") + m); }
    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* s) {
        const char* q = p_;
        for (; *s; ++s, ++q)
            if (q >= e_ || *q != *s) return false;
        p_ = q;
        return true;
    }
    Value value() {
        ws();
        if (p_ >= e_) err("unexpected end");
        if (++depth_ > 256) err("nesting too deep");
        Value v;
        const char c = *p_;
        if (c == '{') {
            v.kind = Value::Object;
            ++p_;
            ws();
            if (p_ < e_ && *p_ == '}') {
                ++p_;
            } else {
                for (;;) {
                    ws();
                    if (p_ >= e_ || *p_ != '"') err("expected a key");
                    std::string k = string();
                    ws();
                    if (p_ >= e_ || *p_ != ':') err("expected ':'");
                    ++p_;
                    v.obj[k] = value();
                    ws();
                    if (p_ < e_ && *p_ == ',') { ++p_; continue; }
                    if (p_ < e_ && *p_ == '}') { ++p_; break; }
                    err("expected ',' or '}'");
                }
            }
        } else if (c == '[') {
            v.kind = Value::Array;
            ++p_;
            ws();
            if (p_ < e_ && *p_ == ']') {
                ++p_;
            } else {
                for (;;) {
                    v.arr.push_back(value());
                    ws();
                    if (p_ < e_ && *p_ == ',') { ++p_; continue; }
                    if (p_ < e_ && *p_ == ']') { ++p_; break; }
                    err("expected ',' or ']'");
                }
            }
        } else if (c == '"') {
            v.kind = Value::String;
            v.str = string();
        } else if (lit("true")) {
            v.kind = Value::Bool, v.b = true;
        } else if (lit("false")) {
            v.kind = Value::Bool, v.b = false;
        } else if (lit("null")) {
            v.kind = Value::Null;
        } else {
            v = number();
        }
        --depth_;
        return v;
    }
    Value number() {
        const char* s = p_;
        bool integer = true;
        if (p_ < e_ && (*p_ == '-' || *p_ == '+')) ++p_;
        while (p_ < e_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '-' ||
                           *p_ == '+')) {
            if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') integer = false;
            ++p_;
        }
        if (p_ == s) err("bad value");
        std::string t(s, p_);
        Value v;
        v.kind = Value::Number;
        char* end = nullptr;
        v.num = std::strtod(t.c_str(), &end);
        if (!end || *end) err("bad number");
        if (integer) {
            v.is_int = true;
            v.inum = std::strtoll(t.c_str(), nullptr, 10);
        }
        return v;
    }
    static void utf8(std::string& o, uint32_t cp) {
        if (cp < 0x80) o += char(cp);
        else if (cp < 0x800) o += char(0xC0 | (cp >> 6)), o += char(0x80 | (cp & 0x3F));
        else if (cp < 0x10000)
            o += char(0xE0 | (cp >> 12)), o += char(0x80 | ((cp >> 6) & 0x3F)), o += char(0x80 | (cp & 0x3F));
        else
            o += char(0xF0 | (cp >> 18)), o += char(0x80 | ((cp >> 12) & 0x3F)), o += char(0x80 | ((cp >> 6) & 0x3F)),
                o += char(0x80 | (cp & 0x3F));
    }
    uint32_t hex4() {
        if (e_ - p_ < 4) err("bad \\u escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) {
            const char h = *p_++;
            v <<= 4;
            if (h >= '0' && h <= '9') v |= h - '0';
            else if (h >= 'a' && h <= 'f') v |= h - 'a' + 10;
            else if (h >= 'A' && h <= 'F') v |= h - 'A' + 10;
            else err("bad \\u escape");
        }
        return v;
    }
    std::string string() {
        ++p_;  // opening quote
        std::string o;
        while (p_ < e_ && *p_ != '"') {
            char c = *p_++;
            if (c != '\\') {
                o += c;
                continue;
            }
            if (p_ >= e_) err("bad escape");
            c = *p_++;
            switch (c) {
                case '"': o += '"'; break;
                case '\\': o += '\\'; break;
                case '/': o += '/'; break;
                case 'b': o += '\b'; break;
                case 'f': o += '\f'; break;
                case 'n': o += '\n'; break;
                case 'r': o += '\r'; break;
                case 't': o += '\t'; break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00 && e_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                        p_ += 2;
                        const uint32_t lo = hex4();
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(o, cp);
                    break;
                }
                default: err("bad escape");
            }
        }
        if (p_ >= e_) err("unterminated string");
        ++p_;
        return o;
    }
};

inline Value parse(const std::string& s) { return Parser(s.data(), s.data() + s.size()).parse_document(); }
inline Value parse(const char* b, const char* e) { return Parser(b, e).parse_document(); }

}  // namespace vb::json
