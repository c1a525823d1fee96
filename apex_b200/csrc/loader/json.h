// json.h -- a small JSON reader for the packed model's manifest.json: objects, arrays, strings
// (with \" \\ \/ \b \f \n \r \t and \uXXXX escapes), numbers (kept as int64 when integral, also
// as double), true / false / null.  Enough for the manifest the packer writes; errors throw
// std::runtime_error with the byte offset.
#pragma once

#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace apex {
namespace json {

struct Value {
    enum class Kind { Null, Bool, Number, String, Array, Object } kind = Kind::Null;
    bool b = false;
    double num = 0.0;
    int64_t integer = 0;
    bool is_integer = false;
    std::string str;
    std::vector<Value> arr;
    std::map<std::string, Value> obj;

    bool has(const std::string &key) const { return kind == Kind::Object && obj.count(key) != 0; }
    const Value &at(const std::string &key) const {
        if (kind != Kind::Object) throw std::runtime_error("json: '" + key + "' looked up in a non-object");
        auto it = obj.find(key);
        if (it == obj.end()) throw std::runtime_error("json: missing key '" + key + "'");
        return it->second;
    }
    const Value &at(size_t i) const {
        if (kind != Kind::Array || i >= arr.size()) throw std::runtime_error("json: array index out of range");
        return arr[i];
    }
    int64_t as_int() const {
        if (kind != Kind::Number || !is_integer) throw std::runtime_error("json: expected an integer");
        return integer;
    }
    uint64_t as_u64() const {
        const int64_t v = as_int();
        if (v < 0) throw std::runtime_error("json: expected a non-negative integer");
        return static_cast<uint64_t>(v);
    }
    double as_double() const {
        if (kind != Kind::Number) throw std::runtime_error("json: expected a number");
        return num;
    }
    bool as_bool() const {
        if (kind != Kind::Bool) throw std::runtime_error("json: expected true or false");
        return b;
    }
    const std::string &as_string() const {
        if (kind != Kind::String) throw std::runtime_error("json: expected a string");
        return str;
    }
    const std::vector<Value> &as_array() const {
        if (kind != Kind::Array) throw std::runtime_error("json: expected an array");
        return arr;
    }
};

class Parser {
  public:
    explicit Parser(const std::string &text) : s_(text) {}

    Value parse() {
        Value v = value(0);
        ws();
        if (i_ != s_.size()) error("trailing characters");
        return v;
    }

  private:
    const std::string &s_;
    size_t i_ = 0;

    [[noreturn]] void error(const std::string &what) const {
        throw std::runtime_error("json: " + what + " at byte " + std::to_string(i_));
    }
    void ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
    }
    char peek() {
        ws();
        if (i_ >= s_.size()) error("unexpected end");
        return s_[i_];
    }
    void expect(char c) {
        if (peek() != c) error(std::string("expected '") + c + "'");
        ++i_;
    }
    bool literal(const char *word) {
        size_t n = 0;
        while (word[n]) ++n;
        if (s_.compare(i_, n, word) == 0) {
            i_ += n;
            return true;
        }
        return false;
    }

    Value value(int depth) {
        if (depth > 64) error("nesting too deep");
        Value v;
        const char c = peek();
        if (c == '{') {
            v.kind = Value::Kind::Object;
            ++i_;
            if (peek() == '}') {
                ++i_;
                return v;
            }
            for (;;) {
                if (peek() != '"') error("expected a key");
                std::string key = string();
                expect(':');
                v.obj[key] = value(depth + 1);
                const char d = peek();
                ++i_;
                if (d == '}') break;
                if (d != ',') error("expected ',' or '}'");
            }
        } else if (c == '[') {
            v.kind = Value::Kind::Array;
            ++i_;
            if (peek() == ']') {
                ++i_;
                return v;
            }
            for (;;) {
                v.arr.push_back(value(depth + 1));
                const char d = peek();
                ++i_;
                if (d == ']') break;
                if (d != ',') error("expected ',' or ']'");
            }
        } else if (c == '"') {
            v.kind = Value::Kind::String;
            v.str = string();
        } else if (literal("true")) {
            v.kind = Value::Kind::Bool;
            v.b = true;
        } else if (literal("false")) {
            v.kind = Value::Kind::Bool;
        } else if (literal("null")) {
            v.kind = Value::Kind::Null;
        } else {
            number(v);
        }
        return v;
    }

    void number(Value &v) {
        const size_t start = i_;
        if (i_ < s_.size() && (s_[i_] == '-' || s_[i_] == '+')) ++i_;
        bool integral = true;
        while (i_ < s_.size()) {
            const char c = s_[i_];
            if (c >= '0' && c <= '9') {
                ++i_;
            } else if (c == '.' || c == 'e' || c == 'E' || c == '-' || c == '+') {
                integral = false;
                ++i_;
            } else {
                break;
            }
        }
        if (i_ == start) error("unexpected character");
        const std::string tok = s_.substr(start, i_ - start);
        char *end = nullptr;
        v.kind = Value::Kind::Number;
        v.num = std::strtod(tok.c_str(), &end);
        if (!end || *end) error("bad number '" + tok + "'");
        if (integral) {
            errno = 0;
            v.integer = std::strtoll(tok.c_str(), &end, 10);
            v.is_integer = errno == 0 && end && !*end;
        }
    }

    static void utf8(std::string &out, uint32_t cp) {
        if (cp < 0x80) {
            out += static_cast<char>(cp);
        } else if (cp < 0x800) {
            out += static_cast<char>(0xC0 | (cp >> 6));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += static_cast<char>(0xE0 | (cp >> 12));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else {
            out += static_cast<char>(0xF0 | (cp >> 18));
            out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        }
    }

    uint32_t hex4() {
        if (i_ + 4 > s_.size()) error("short \\u escape");
        uint32_t v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = s_[i_++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= c - '0';
            else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
            else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
            else error("bad \\u escape");
        }
        return v;
    }

    std::string string() {
        expect('"');
        std::string out;
        for (;;) {
            if (i_ >= s_.size()) error("unterminated string");
            const char c = s_[i_++];
            if (c == '"') break;
            if (c != '\\') {
                out += c;
                continue;
            }
            if (i_ >= s_.size()) error("unterminated escape");
            const char e = s_[i_++];
            switch (e) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00 && i_ + 1 < s_.size() && s_[i_] == '\\' && s_[i_ + 1] == 'u') {
                        i_ += 2;
                        const uint32_t lo = hex4();
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(out, cp);
                    break;
                }
                default: error("bad escape");
            }
        }
        return out;
    }
};

inline Value parse(const std::string &text) { return Parser(text).parse(); }

}  // namespace json
}  // namespace apex
