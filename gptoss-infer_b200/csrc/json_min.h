// Minimal JSON reader for checkpoint metadata (config.json, generation_config.json, safetensors headers and
// index files): objects, arrays, strings (with the common escapes), numbers, true, false and null. Values are parsed
// into a small tree; lookups throw with the missing key's name.
#pragma once
#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace gpt {
namespace json {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Value> arr;
    std::map<std::string, Value> obj;

    bool has(const std::string& k) const { return kind == Object && obj.count(k) != 0; }
    const Value& at(const std::string& k) const {
        if (kind != Object) throw std::runtime_error("json: not an object (looking up '" + k + "')");
        auto it = obj.find(k);
        if (it == obj.end()) throw std::runtime_error("json: missing key '" + k + "'");
        return it->second;
    }
    double number() const {
        if (kind != Number) throw std::runtime_error("json: not a number");
        return num;
    }
    long long integer() const { return static_cast<long long>(number()); }
    bool boolean() const {
        if (kind != Bool) throw std::runtime_error("json: not a boolean");
        return b;
    }
    const std::string& string() const {
        if (kind != String) throw std::runtime_error("json: not a string");
        return str;
    }
};

class Parser {
  public:
    explicit Parser(const std::string& text) : s_(text) {}
    Value parse() {
        Value v = value();
        skip();
        if (i_ != s_.size()) fail("trailing characters");
        return v;
    }

  private:
    const std::string& s_;
    size_t i_ = 0;

    [[noreturn]] void fail(const char* what) const {
        throw std::runtime_error(std::string("json: ") + what + " at offset " + std::to_string(i_));
    }
    void skip() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
    }
    char peek() {
        skip();
        if (i_ >= s_.size()) fail("unexpected end");
        return s_[i_];
    }
    void expect(char c) {
        if (peek() != c) fail("unexpected character");
        ++i_;
    }
    bool word(const char* w) {
        size_t n = 0;
        while (w[n]) ++n;
        if (s_.compare(i_, n, w) != 0) return false;
        i_ += n;
        return true;
    }
    Value value() {
        const char c = peek();
        Value v;
        if (c == '{') {
            v.kind = Value::Object;
            ++i_;
            if (peek() == '}') { ++i_; return v; }
            while (true) {
                if (peek() != '"') fail("expected a key");
                std::string k = string_body();
                expect(':');
                v.obj.emplace(std::move(k), value());
                const char d = peek();
                ++i_;
                if (d == '}') break;
                if (d != ',') fail("expected ',' or '}'");
            }
        } else if (c == '[') {
            v.kind = Value::Array;
            ++i_;
            if (peek() == ']') { ++i_; return v; }
            while (true) {
                v.arr.push_back(value());
                const char d = peek();
                ++i_;
                if (d == ']') break;
                if (d != ',') fail("expected ',' or ']'");
            }
        } else if (c == '"') {
            v.kind = Value::String;
            v.str = string_body();
        } else if (word("true")) {
            v.kind = Value::Bool;
            v.b = true;
        } else if (word("false")) {
            v.kind = Value::Bool;
        } else if (word("null")) {
            v.kind = Value::Null;
        } else {
            const char* start = s_.c_str() + i_;
            char* end = nullptr;
            v.num = std::strtod(start, &end);
            if (end == start) fail("bad value");
            v.kind = Value::Number;
            i_ += size_t(end - start);
        }
        return v;
    }
    std::string string_body() {
        ++i_;                                                    // opening quote
        std::string out;
        while (i_ < s_.size() && s_[i_] != '"') {
            char c = s_[i_++];
            if (c == '\\') {
                if (i_ >= s_.size()) fail("bad escape");
                const char e = s_[i_++];
                switch (e) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {                                  // keep ASCII, replace the rest (names are ASCII)
                        if (i_ + 4 > s_.size()) fail("bad \\u escape");
                        const unsigned cp = unsigned(std::strtoul(s_.substr(i_, 4).c_str(), nullptr, 16));
                        out += cp < 128 ? char(cp) : '?';
                        i_ += 4;
                        break;
                    }
                    default: out += e;
                }
            } else {
                out += c;
            }
        }
        if (i_ >= s_.size()) fail("unterminated string");
        ++i_;
        return out;
    }
};

inline Value parse(const std::string& text) { return Parser(text).parse(); }

}  // namespace json
}  // namespace gpt
