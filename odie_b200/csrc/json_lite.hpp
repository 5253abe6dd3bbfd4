// Minimal JSON reader/writer for the runtime's configuration strings.
// Supports objects, arrays, strings, numbers (kept as both int64 and double),
// true/false/null.  Numbers keep their integer value exactly when written as
// integers, so 64-bit device pointers survive the round trip.
#pragma once
#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace odie {

struct Json {
    enum Type { NUL, BOOL, NUMBER, STRING, ARRAY, OBJECT } type = NUL;
    bool boolean = false;
    bool integral = false;
    long long integer = 0;
    unsigned long long uinteger = 0;
    double number = 0;
    std::string text;
    std::vector<Json> items;
    std::map<std::string, Json> fields;

    bool contains(const std::string& key) const { return type == OBJECT && fields.count(key); }
    const Json& at(const std::string& key) const {
        auto it = fields.find(key);
        if (type != OBJECT || it == fields.end()) throw std::invalid_argument("missing configuration key: " + key);
        return it->second;
    }
    long long as_int() const {
        if (type == BOOL) return boolean;
        if (type != NUMBER) throw std::invalid_argument("expected a number");
        return integral ? integer : (long long)number;
    }
    unsigned long long as_u64() const {
        if (type != NUMBER) throw std::invalid_argument("expected a number");
        return integral ? uinteger : (unsigned long long)number;
    }
    double as_double() const {
        if (type == BOOL) return boolean;
        if (type != NUMBER) throw std::invalid_argument("expected a number");
        return number;
    }
    long long value(const std::string& key, long long fallback) const {
        return contains(key) ? at(key).as_int() : fallback;
    }
    double value_double(const std::string& key, double fallback) const {
        return contains(key) ? at(key).as_double() : fallback;
    }
};

class JsonParser {
  public:
    explicit JsonParser(const std::string& s) : s_(s) {}
    Json parse() {
        Json v = value();
        skip();
        if (p_ != s_.size()) fail("trailing characters");
        return v;
    }

  private:
    const std::string& s_;
    size_t p_ = 0;
    [[noreturn]] void fail(const char* why) { throw std::invalid_argument(std::string("invalid JSON: ") + why); }
    void skip() {
        while (p_ < s_.size() && (s_[p_] == ' ' || s_[p_] == '\n' || s_[p_] == '\t' || s_[p_] == '\r')) ++p_;
    }
    bool eat(char c) {
        skip();
        if (p_ < s_.size() && s_[p_] == c) { ++p_; return true; }
        return false;
    }
    std::string str() {
        if (!eat('"')) fail("expected string");
        std::string out;
        while (p_ < s_.size() && s_[p_] != '"') {
            char c = s_[p_++];
            if (c == '\\' && p_ < s_.size()) {
                char e = s_[p_++];
                if (e == 'n') out += '\n';
                else if (e == 't') out += '\t';
                else if (e == 'u') { p_ += 4; out += '?'; }
                else out += e;
            } else {
                out += c;
            }
        }
        if (p_ >= s_.size()) fail("unterminated string");
        ++p_;
        return out;
    }
    Json value() {
        skip();
        if (p_ >= s_.size()) fail("unexpected end");
        Json v;
        char c = s_[p_];
        if (c == '{') {
            ++p_;
            v.type = Json::OBJECT;
            if (eat('}')) return v;
            do {
                std::string key = str();
                if (!eat(':')) fail("expected ':'");
                v.fields[key] = value();
            } while (eat(','));
            if (!eat('}')) fail("expected '}'");
        } else if (c == '[') {
            ++p_;
            v.type = Json::ARRAY;
            if (eat(']')) return v;
            do { v.items.push_back(value()); } while (eat(','));
            if (!eat(']')) fail("expected ']'");
        } else if (c == '"') {
            v.type = Json::STRING;
            v.text = str();
        } else if (s_.compare(p_, 4, "true") == 0) {
            p_ += 4; v.type = Json::BOOL; v.boolean = true;
        } else if (s_.compare(p_, 5, "false") == 0) {
            p_ += 5; v.type = Json::BOOL;
        } else if (s_.compare(p_, 4, "null") == 0) {
            p_ += 4;
        } else {
            size_t start = p_;
            bool integral = true;
            if (s_[p_] == '-' || s_[p_] == '+') ++p_;
            while (p_ < s_.size() && (isdigit((unsigned char)s_[p_]) || s_[p_] == '.' || s_[p_] == 'e' || s_[p_] == 'E' ||
                                      s_[p_] == '-' || s_[p_] == '+')) {
                if (s_[p_] == '.' || s_[p_] == 'e' || s_[p_] == 'E') integral = false;
                ++p_;
            }
            if (start == p_) fail("unexpected character");
            std::string token = s_.substr(start, p_ - start);
            v.type = Json::NUMBER;
            v.number = strtod(token.c_str(), nullptr);
            v.integral = integral;
            if (integral) {
                if (token[0] == '-') { v.integer = strtoll(token.c_str(), nullptr, 10); v.uinteger = (unsigned long long)v.integer; }
                else { v.uinteger = strtoull(token.c_str(), nullptr, 10); v.integer = (long long)v.uinteger; }
            }
        }
        return v;
    }
};

inline Json parse_json(const char* text) {
    if (!text) throw std::invalid_argument("null configuration string");
    std::string s(text);
    return JsonParser(s).parse();
}

}  // namespace odie
