// model_compile.cpp -- JSON model documents -> geo_cycle model IR
// ("geo_model_ir=8"), in the library (geo_b200_model_compile) and behind the
// geo_cycle_b200 command (compile | validate), so the model path from document
// to trained parameters has no Python in it.
//
// Contract with the reference's compiler (tools/geo_model.py): the accepted
// documents, the order in which rules are checked (the first failing rule's
// message is the one reported), the messages, the IR line grammar and the
// `random:` initialiser stream are the reference's, so a document compiles to
// the same IR bytes with either and is rejected with the same message. The
// implementation is this file's own:
//
//  * Document: a JSON reader with the semantics of Python's json module, which
//    the reference uses (NaN / Infinity literals accepted, integers of any
//    length kept exact, a repeated key keeps its first position and its last
//    value, the same syntax-error wording and positions), over the text as
//    Python reads it (UTF-8, universal newlines).
//  * Rules: tables of fields (name, default, type rule, message label) walked in
//    order; the node ops, constraints and optimizers are tables of codes.
//  * Integers: arbitrary length (the document's seed, the basis index and the
//    initialiser seed may be any integer), as magnitude words.
//  * `random:` initialisers: the Mersenne Twister MT19937 of Matsumoto and
//    Nishimura (init_by_array seeding with the 32-bit words of |seed|, 53-bit
//    doubles from two outputs) -- the generator behind Python's random.Random,
//    which the reference seeds with (seed << 32) ^ (sum of the name's code
//    points) and draws with uniform(-scale, scale).
//
// A node op, constraint or optimizer type given as a JSON array or object is
// rejected here with the rule's message; the reference's compiler stops with a
// Python TypeError there (such values cannot be looked up in its tables).
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "geo/geo_cycle_b200.h"

namespace {

// ---- arbitrary-length integers ------------------------------------------------
struct BigInt {
    bool negative = false;
    std::vector<uint32_t> words;  // magnitude, little-endian; empty = 0

    bool zero() const { return words.empty(); }
    void trim() {
        while (!words.empty() && words.back() == 0) words.pop_back();
        if (words.empty()) negative = false;
    }
    void mul_add(uint32_t m, uint32_t a) {
        uint64_t carry = a;
        for (uint32_t &w : words) {
            const uint64_t v = (uint64_t)w * m + carry;
            w = (uint32_t)v;
            carry = v >> 32;
        }
        if (carry) words.push_back((uint32_t)carry);
    }
    static BigInt from_digits(const std::string &digits, bool neg) {
        BigInt b;
        for (char c : digits) b.mul_add(10, (uint32_t)(c - '0'));
        b.negative = neg;
        b.trim();
        return b;
    }
    std::string decimal() const {
        if (words.empty()) return "0";
        std::vector<uint32_t> w = words;
        std::string out;
        while (!w.empty()) {
            uint64_t rem = 0;
            for (size_t i = w.size(); i-- > 0;) {
                const uint64_t cur = (rem << 32) | w[i];
                w[i] = (uint32_t)(cur / 1000000000u);
                rem = cur % 1000000000u;
            }
            while (!w.empty() && w.back() == 0) w.pop_back();
            char buf[16];
            snprintf(buf, sizeof buf, w.empty() ? "%u" : "%09u", (unsigned)rem);
            out.insert(0, buf);
        }
        return negative ? "-" + out : out;
    }
    int compare_small(int64_t v) const {  // sign of (this - v), |v| < 2^63
        const bool vneg = v < 0;
        const uint64_t mag = vneg ? (uint64_t)(-(v + 1)) + 1 : (uint64_t)v;
        if (negative != vneg) return negative ? -1 : (zero() && mag == 0 ? 0 : 1);
        int c;
        if (words.size() > 2) c = 1;
        else {
            const uint64_t me = (words.size() > 0 ? words[0] : 0) | ((uint64_t)(words.size() > 1 ? words[1] : 0) << 32);
            c = me > mag ? 1 : (me < mag ? -1 : 0);
        }
        return negative ? -c : c;
    }
    double to_double() const {  // correctly rounded, via the decimal string
        return strtod(decimal().c_str(), nullptr);
    }
};

// ---- JSON values with Python's json semantics -----------------------------------
struct JValue;
using JPtr = std::shared_ptr<JValue>;
enum class JKind { Null, Bool, Int, Float, String, Array, Object };

struct JValue {
    JKind kind = JKind::Null;
    bool boolean = false;
    BigInt integer;
    double number = 0.0;
    std::u32string text;
    std::vector<JPtr> items;
    std::vector<std::pair<std::u32string, JPtr>> members;  // first position, last value

    const JValue *get(const char *key) const {
        for (const auto &m : members)
            if (m.first.size() == strlen(key) && std::equal(m.first.begin(), m.first.end(), key,
                                                             [](char32_t a, char b) { return a == (unsigned char)b; }))
                return m.second.get();
        return nullptr;
    }
    bool has(const char *key) const { return get(key) != nullptr; }
};

std::string utf8(const std::u32string &s) {
    std::string o;
    for (char32_t c : s) {
        if (c < 0x80) o += (char)c;
        else if (c < 0x800) {
            o += (char)(0xC0 | (c >> 6));
            o += (char)(0x80 | (c & 0x3F));
        } else if (c < 0x10000) {
            o += (char)(0xE0 | (c >> 12));
            o += (char)(0x80 | ((c >> 6) & 0x3F));
            o += (char)(0x80 | (c & 0x3F));
        } else {
            o += (char)(0xF0 | (c >> 18));
            o += (char)(0x80 | ((c >> 12) & 0x3F));
            o += (char)(0x80 | ((c >> 6) & 0x3F));
            o += (char)(0x80 | (c & 0x3F));
        }
    }
    return o;
}

std::u32string widen(const std::string &s) { return std::u32string(s.begin(), s.end()); }

struct Failure {
    std::string message;
};

// Recursive-descent reader over code points; errors carry Python's wording and
// its "line L column C (char P)" position.
class Reader {
  public:
    explicit Reader(const std::u32string &t) : t_(t) {}

    JPtr document() {
        size_t i = skip(0);
        JPtr v = value(i, &i);
        i = skip(i);
        if (i != t_.size()) fail("Extra data", i);
        return v;
    }

  private:
    const std::u32string &t_;

    [[noreturn]] void fail(const char *what, size_t pos) const {
        size_t line = 1, last_nl = (size_t)-1;
        for (size_t k = 0; k < pos && k < t_.size(); ++k)
            if (t_[k] == U'\n') {
                ++line;
                last_nl = k;
            }
        const size_t col = last_nl == (size_t)-1 ? pos + 1 : pos - last_nl;
        char buf[160];
        snprintf(buf, sizeof buf, "%s: line %zu column %zu (char %zu)", what, line, col, pos);
        throw Failure{buf};
    }
    size_t skip(size_t i) const {
        while (i < t_.size() && (t_[i] == U' ' || t_[i] == U'\t' || t_[i] == U'\n' || t_[i] == U'\r')) ++i;
        return i;
    }
    bool at(size_t i, const char *lit) const {
        for (size_t k = 0; lit[k]; ++k)
            if (i + k >= t_.size() || t_[i + k] != (char32_t)lit[k]) return false;
        return true;
    }
    JPtr value(size_t i, size_t *end) {
        if (i >= t_.size()) fail("Expecting value", i);
        const char32_t c = t_[i];
        auto v = std::make_shared<JValue>();
        if (c == U'"') {
            v->kind = JKind::String;
            v->text = string(i + 1, end);
        } else if (c == U'{') {
            object(i + 1, end, *v);
        } else if (c == U'[') {
            array(i + 1, end, *v);
        } else if (at(i, "null")) {
            *end = i + 4;
        } else if (at(i, "true") || at(i, "false")) {
            v->kind = JKind::Bool;
            v->boolean = c == U't';
            *end = i + (v->boolean ? 4 : 5);
        } else if (at(i, "NaN")) {
            v->kind = JKind::Float;
            v->number = NAN;
            *end = i + 3;
        } else if (at(i, "Infinity")) {
            v->kind = JKind::Float;
            v->number = INFINITY;
            *end = i + 8;
        } else if (at(i, "-Infinity")) {
            v->kind = JKind::Float;
            v->number = -INFINITY;
            *end = i + 9;
        } else if (!number(i, end, *v)) {
            fail("Expecting value", i);
        }
        return v;
    }
    // -?(0|[1-9][0-9]*)(\.[0-9]+)?([eE][-+]?[0-9]+)?
    bool number(size_t i, size_t *end, JValue &v) {
        size_t k = i;
        const bool neg = k < t_.size() && t_[k] == U'-';
        if (neg) ++k;
        auto digit = [&](size_t p) { return p < t_.size() && t_[p] >= U'0' && t_[p] <= U'9'; };
        if (!digit(k)) return false;
        const size_t int_start = k;
        if (t_[k] == U'0') ++k;
        else
            while (digit(k)) ++k;
        const size_t int_end = k;
        bool is_float = false;
        if (k < t_.size() && t_[k] == U'.' && digit(k + 1)) {
            is_float = true;
            k += 1;
            while (digit(k)) ++k;
        }
        if (k < t_.size() && (t_[k] == U'e' || t_[k] == U'E')) {
            size_t e = k + 1;
            if (e < t_.size() && (t_[e] == U'+' || t_[e] == U'-')) ++e;
            if (digit(e)) {
                is_float = true;
                k = e;
                while (digit(k)) ++k;
            }
        }
        const std::string lexeme = utf8(t_.substr(i, k - i));
        if (is_float) {
            v.kind = JKind::Float;
            v.number = strtod(lexeme.c_str(), nullptr);
        } else {
            v.kind = JKind::Int;
            v.integer = BigInt::from_digits(utf8(t_.substr(int_start, int_end - int_start)), neg);
        }
        *end = k;
        return true;
    }
    std::u32string string(size_t i, size_t *end) {
        const size_t begin = i - 1;
        std::u32string out;
        for (;;) {
            if (i >= t_.size()) fail("Unterminated string starting at", begin);
            const char32_t c = t_[i];
            if (c == U'"') {
                *end = i + 1;
                return out;
            }
            if (c < 0x20) fail("Invalid control character at", i);
            if (c != U'\\') {
                out += c;
                ++i;
                continue;
            }
            if (i + 1 >= t_.size()) fail("Unterminated string starting at", begin);
            const char32_t e = t_[i + 1];
            switch (e) {
                case U'"': out += U'"'; break;
                case U'\\': out += U'\\'; break;
                case U'/': out += U'/'; break;
                case U'b': out += U'\b'; break;
                case U'f': out += U'\f'; break;
                case U'n': out += U'\n'; break;
                case U'r': out += U'\r'; break;
                case U't': out += U'\t'; break;
                case U'u': {
                    char32_t u = hex4(i + 2, i + 1);  // errors point at the 'u'

                    i += 6;
                    if (u >= 0xD800 && u <= 0xDBFF && at(i, "\\u")) {
                        const char32_t lo = hex4(i + 2, i + 1);
                        if (lo >= 0xDC00 && lo <= 0xDFFF) {
                            u = 0x10000 + ((u - 0xD800) << 10) + (lo - 0xDC00);
                            i += 6;
                        }
                    }
                    out += u;
                    continue;
                }
                default: fail("Invalid \\escape", i);
            }
            i += 2;
        }
    }
    char32_t hex4(size_t p, size_t escape_pos) const {
        char32_t v = 0;
        for (size_t k = 0; k < 4; ++k) {
            if (p + k >= t_.size()) fail("Invalid \\uXXXX escape", escape_pos);
            const char32_t c = t_[p + k];
            int d = c >= U'0' && c <= U'9' ? (int)(c - U'0')
                    : c >= U'a' && c <= U'f' ? (int)(c - U'a' + 10)
                    : c >= U'A' && c <= U'F' ? (int)(c - U'A' + 10) : -1;
            if (d < 0) fail("Invalid \\uXXXX escape", escape_pos);
            v = v * 16 + (char32_t)d;
        }
        return v;
    }
    void object(size_t i, size_t *end, JValue &v) {
        v.kind = JKind::Object;
        i = skip(i);
        if (i < t_.size() && t_[i] == U'}') {
            *end = i + 1;
            return;
        }
        for (;;) {
            if (i >= t_.size() || t_[i] != U'"') fail("Expecting property name enclosed in double quotes", i);
            size_t k;
            std::u32string key = string(i + 1, &k);
            k = skip(k);
            if (k >= t_.size() || t_[k] != U':') fail("Expecting ':' delimiter", k);
            k = skip(k + 1);
            JPtr item = value(k, &k);
            bool replaced = false;
            for (auto &m : v.members)
                if (m.first == key) {
                    m.second = item;
                    replaced = true;
                }
            if (!replaced) v.members.emplace_back(std::move(key), item);
            k = skip(k);
            if (k < t_.size() && t_[k] == U'}') {
                *end = k + 1;
                return;
            }
            if (k >= t_.size() || t_[k] != U',') fail("Expecting ',' delimiter", k);
            i = skip(k + 1);
        }
    }
    void array(size_t i, size_t *end, JValue &v) {
        v.kind = JKind::Array;
        i = skip(i);
        if (i < t_.size() && t_[i] == U']') {
            *end = i + 1;
            return;
        }
        for (;;) {
            size_t k;
            v.items.push_back(value(i, &k));
            k = skip(k);
            if (k < t_.size() && t_[k] == U']') {
                *end = k + 1;
                return;
            }
            if (k >= t_.size() || t_[k] != U',') fail("Expecting ',' delimiter", k);
            i = skip(k + 1);
        }
    }
};

// UTF-8 text -> code points with universal newlines, as Python's text read does.
std::u32string decode_text(const std::string &bytes) {
    std::u32string out;
    size_t i = 0;
    auto bad = [&](size_t pos, const char *why) {
        char buf[128];
        snprintf(buf, sizeof buf, "'utf-8' codec can't decode byte 0x%02x in position %zu: %s",
                 (unsigned char)bytes[pos], pos, why);
        throw Failure{buf};
    };
    while (i < bytes.size()) {
        const unsigned char c = (unsigned char)bytes[i];
        char32_t cp;
        size_t n;
        if (c < 0x80) {
            cp = c;
            n = 1;
        } else if (c >= 0xC2 && c <= 0xDF) {
            cp = c & 0x1F;
            n = 2;
        } else if (c >= 0xE0 && c <= 0xEF) {
            cp = c & 0x0F;
            n = 3;
        } else if (c >= 0xF0 && c <= 0xF4) {
            cp = c & 0x07;
            n = 4;
        } else {
            bad(i, "invalid start byte");
        }
        for (size_t k = 1; k < n; ++k) {
            if (i + k >= bytes.size()) bad(i, "unexpected end of data");
            const unsigned char d = (unsigned char)bytes[i + k];
            const bool ok = (d & 0xC0) == 0x80 && !(k == 1 && ((c == 0xE0 && d < 0xA0) || (c == 0xED && d > 0x9F) ||
                                                              (c == 0xF0 && d < 0x90) || (c == 0xF4 && d > 0x8F)));
            if (!ok) bad(i, "invalid continuation byte");
            cp = (cp << 6) | (d & 0x3F);
        }
        i += n;
        if (cp == U'\r') {
            out += U'\n';
            if (i < bytes.size() && bytes[i] == '\n') ++i;
        } else {
            out += cp;
        }
    }
    return out;
}

// ---- Python text forms used in messages ------------------------------------------
std::string py_repr_str(const std::u32string &s) {
    const bool has_single = s.find(U'\'') != std::u32string::npos;
    const bool has_double = s.find(U'"') != std::u32string::npos;
    const char32_t q = has_single && !has_double ? U'"' : U'\'';
    std::u32string o(1, q);
    for (char32_t c : s) {
        if (c == q || c == U'\\') {
            o += U'\\';
            o += c;
        } else if (c == U'\n') o += U"\\n";
        else if (c == U'\r') o += U"\\r";
        else if (c == U'\t') o += U"\\t";
        else if (c < 0x20 || c == 0x7F || (c >= 0x80 && c < 0xA0)) {
            char buf[8];
            snprintf(buf, sizeof buf, "\\x%02x", (unsigned)c);
            o += widen(buf);
        } else {
            o += c;
        }
    }
    o += q;
    return utf8(o);
}

// repr(float): the shortest digits that read back exactly, in Python's layout.
std::string py_float(double v) {
    if (isnan(v)) return "nan";
    if (isinf(v)) return v > 0 ? "inf" : "-inf";
    char buf[64];
    int prec = 1;
    for (; prec <= 17; ++prec) {
        snprintf(buf, sizeof buf, "%.*e", prec - 1, v);
        if (strtod(buf, nullptr) == v) break;
    }
    // buf = d.ddde[+-]XX: split into digits and decimal exponent
    std::string s = buf, digits;
    const bool neg = s[0] == '-';
    const size_t e = s.find('e');
    for (size_t k = neg ? 1 : 0; k < e; ++k)
        if (s[k] != '.') digits += s[k];
    while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
    const int exp10 = atoi(s.c_str() + e + 1);
    std::string out;
    if (exp10 < -4 || exp10 >= 16) {
        out = digits.substr(0, 1);
        if (digits.size() > 1) out += "." + digits.substr(1);
        snprintf(buf, sizeof buf, "e%c%02d", exp10 < 0 ? '-' : '+', exp10 < 0 ? -exp10 : exp10);
        out += buf;
    } else if (exp10 < 0) {
        out = "0." + std::string((size_t)(-exp10 - 1), '0') + digits;
    } else if ((int)digits.size() <= exp10 + 1) {
        out = digits + std::string((size_t)(exp10 + 1 - (int)digits.size()), '0') + ".0";
    } else {
        out = digits.substr(0, (size_t)exp10 + 1) + "." + digits.substr((size_t)exp10 + 1);
    }
    return neg ? "-" + out : out;
}

std::string py_str(const JValue &v, bool top = true) {
    switch (v.kind) {
        case JKind::Null: return "None";
        case JKind::Bool: return v.boolean ? "True" : "False";
        case JKind::Int: return v.integer.decimal();
        case JKind::Float: return py_float(v.number);
        case JKind::String: return top ? utf8(v.text) : py_repr_str(v.text);
        case JKind::Array: {
            std::string o = "[";
            for (size_t k = 0; k < v.items.size(); ++k) o += (k ? ", " : "") + py_str(*v.items[k], false);
            return o + "]";
        }
        case JKind::Object: {
            std::string o = "{";
            for (size_t k = 0; k < v.members.size(); ++k)
                o += (k ? ", " : "") + py_repr_str(v.members[k].first) + ": " + py_str(*v.members[k].second, false);
            return o + "}";
        }
    }
    return "";
}

// ---- Python's float() and int() on initialiser fields ----------------------------
bool py_space(char c) { return c == ' ' || (c >= '\t' && c <= '\r'); }

std::string strip(const std::string &s) {
    size_t a = 0, b = s.size();
    while (a < b && py_space(s[a])) ++a;
    while (b > a && py_space(s[b - 1])) --b;
    return s.substr(a, b - a);
}

// Underscores only between digits (PEP 515); returns false otherwise.
bool drop_underscores(const std::string &s, std::string *out) {
    out->clear();
    for (size_t k = 0; k < s.size(); ++k) {
        if (s[k] != '_') {
            *out += s[k];
            continue;
        }
        if (k == 0 || k + 1 >= s.size() || !isdigit((unsigned char)s[k - 1]) || !isdigit((unsigned char)s[k + 1]))
            return false;
    }
    return true;
}

double py_float_of(const std::string &raw) {
    const std::string bad = "could not convert string to float: " + py_repr_str(widen(raw));
    std::string s = strip(raw), t;
    if (!drop_underscores(s, &t) || t.empty()) throw Failure{bad};
    std::string lower;
    for (char c : t) lower += (char)tolower((unsigned char)c);
    const size_t sign = (lower[0] == '+' || lower[0] == '-') ? 1 : 0;
    const std::string body = lower.substr(sign);
    if (body == "inf" || body == "infinity") return lower[0] == '-' ? -INFINITY : INFINITY;
    if (body == "nan") return NAN;
    // decimal digits with an optional point and exponent, nothing else
    size_t k = sign;
    bool digits = false;
    while (k < t.size() && isdigit((unsigned char)t[k])) k++, digits = true;
    if (k < t.size() && t[k] == '.') {
        ++k;
        while (k < t.size() && isdigit((unsigned char)t[k])) k++, digits = true;
    }
    if (!digits) throw Failure{bad};
    if (k < t.size() && (t[k] == 'e' || t[k] == 'E')) {
        size_t e = k + 1;
        if (e < t.size() && (t[e] == '+' || t[e] == '-')) ++e;
        if (e >= t.size() || !isdigit((unsigned char)t[e])) throw Failure{bad};
        while (e < t.size() && isdigit((unsigned char)t[e])) ++e;
        k = e;
    }
    if (k != t.size()) throw Failure{bad};
    return strtod(t.c_str(), nullptr);
}

BigInt py_int_of(const std::string &raw) {
    const std::string bad = "invalid literal for int() with base 10: " + py_repr_str(widen(raw));
    std::string s = strip(raw), t;
    if (!drop_underscores(s, &t) || t.empty()) throw Failure{bad};
    const bool neg = t[0] == '-';
    const size_t sign = (t[0] == '+' || t[0] == '-') ? 1 : 0;
    if (sign == t.size()) throw Failure{bad};
    for (size_t k = sign; k < t.size(); ++k)
        if (!isdigit((unsigned char)t[k])) throw Failure{bad};
    return BigInt::from_digits(t.substr(sign), neg);
}

// ---- MT19937 (Matsumoto & Nishimura), seeded like Python's random.Random(int) -------
class Mt19937 {
  public:
    explicit Mt19937(const std::vector<uint32_t> &key) {
        init(19650218u);
        const size_t len = key.size();
        size_t i = 1, j = 0;
        for (size_t k = std::max<size_t>(kN, len); k > 0; --k) {
            s_[i] = (s_[i] ^ ((s_[i - 1] ^ (s_[i - 1] >> 30)) * 1664525u)) + key[j] + (uint32_t)j;
            ++i;
            ++j;
            if (i >= kN) {
                s_[0] = s_[kN - 1];
                i = 1;
            }
            if (j >= len) j = 0;
        }
        for (size_t k = kN - 1; k > 0; --k) {
            s_[i] = (s_[i] ^ ((s_[i - 1] ^ (s_[i - 1] >> 30)) * 1566083941u)) - (uint32_t)i;
            ++i;
            if (i >= kN) {
                s_[0] = s_[kN - 1];
                i = 1;
            }
        }
        s_[0] = 0x80000000u;
        index_ = kN;
    }
    // 53-bit uniform double in [0, 1).
    double unit() {
        const uint32_t a = next() >> 5, b = next() >> 6;
        return (a * 67108864.0 + b) * (1.0 / 9007199254740992.0);
    }

  private:
    static constexpr size_t kN = 624, kM = 397;
    uint32_t s_[kN];
    size_t index_ = kN;

    void init(uint32_t seed) {
        s_[0] = seed;
        for (size_t i = 1; i < kN; ++i) s_[i] = 1812433253u * (s_[i - 1] ^ (s_[i - 1] >> 30)) + (uint32_t)i;
    }
    uint32_t next() {
        if (index_ >= kN) {
            for (size_t k = 0; k < kN; ++k) {
                const uint32_t y = (s_[k] & 0x80000000u) | (s_[(k + 1) % kN] & 0x7fffffffu);
                s_[k] = s_[(k + kM) % kN] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
            }
            index_ = 0;
        }
        uint32_t y = s_[index_++];
        y ^= y >> 11;
        y ^= (y << 7) & 0x9d2c5680u;
        y ^= (y << 15) & 0xefc60000u;
        y ^= y >> 18;
        return y;
    }
};

// Seed words of |(seed << 32) ^ code_sum| (code_sum < 2^32).
std::vector<uint32_t> random_key(const BigInt &seed, uint32_t code_sum) {
    BigInt v;
    v.words.push_back(0);
    v.words.insert(v.words.end(), seed.words.begin(), seed.words.end());
    v.negative = seed.negative;
    if (!v.negative) {
        v.words[0] = code_sum;
    } else if (code_sum != 0) {
        // -(m * 2^32) ^ s for 0 <= s < 2^32 is -(m * 2^32) + s: magnitude m * 2^32 - s
        uint64_t borrow = code_sum;
        for (uint32_t &w : v.words) {
            const uint64_t cur = (uint64_t)w;
            const uint64_t sub = borrow;
            w = (uint32_t)(cur - sub);
            borrow = cur < sub ? 1 : 0;
            if (!borrow) break;
        }
    }
    v.trim();
    std::vector<uint32_t> key = v.words;
    if (key.empty()) key.push_back(0);
    return key;
}

// ---- rule tables -------------------------------------------------------------------
const char *const kRootKeys[] = {"version", "dimension", "signature", "seed",     "nodes",   "loss",
                                 "output",  "state_updates", "optimizer", "training", "dataset", "metadata"};
const char *const kNodeKeys[] = {"name", "op", "inputs", "input", "scalar", "grade", "constraint", "requires_grad",
                                 "init"};

enum Arity { kLeaf, kOneInput, kTwoInputs };
struct OpRule {
    const char *name;
    int code;
    Arity arity;
};
const OpRule kOps[] = {
    {"input", 1, kLeaf},           {"target", 2, kLeaf},           {"parameter", 3, kLeaf},
    {"constant", 4, kLeaf},        {"state", 5, kLeaf},            {"add", 6, kTwoInputs},
    {"scale", 7, kOneInput},       {"gp", 8, kTwoInputs},          {"reverse", 9, kOneInput},
    {"grade_project", 10, kOneInput}, {"grade_involution", 11, kOneInput}, {"clifford_conjugate", 12, kOneInput},
    {"hadamard", 13, kTwoInputs},  {"tanh", 14, kOneInput},        {"sigmoid", 15, kOneInput},
    {"normalize", 16, kOneInput},  {"squared_norm", 17, kOneInput},
};
struct Code {
    const char *name;
    int code;
};
const Code kConstraints[] = {{"none", 0}, {"unit_euclidean", 1}, {"unit_vector_metric", 2}, {"even_versor", 3}};
const Code kOptimizers[] = {{"sgd", 1}, {"adam", 2}};

enum NumberRule { kFinite, kPositive };
struct NumberField {
    const char *key;
    double fallback;
    NumberRule rule;
    const char *label;
};
const NumberField kOptimizerNumbers[] = {{"learning_rate", 0.01, kPositive, "optimizer.learning_rate"},
                                         {"beta1", 0.9, kFinite, "optimizer.beta1"},
                                         {"beta2", 0.999, kFinite, "optimizer.beta2"},
                                         {"epsilon", 1e-8, kPositive, "optimizer.epsilon"}};
struct CountField {
    const char *key;
    const char *label;
};
const CountField kTrainingCounts[] = {{"epochs", "training.epochs"}, {"batch_size", "training.batch_size"}};

[[noreturn]] void reject(const std::string &m) { throw Failure{m}; }

bool is_string(const JValue *v, const char *s) {
    return v != nullptr && v->kind == JKind::String && utf8(v->text) == s;
}

// A number (not a boolean), finite; positive when asked.
double number_of(const JValue &v, const std::string &label, NumberRule rule) {
    double d;
    if (v.kind == JKind::Int) d = v.integer.to_double();
    else if (v.kind == JKind::Float) d = v.number;
    else reject(label + " must be a number");
    if (!isfinite(d)) reject(label + " must be finite");
    if (rule == kPositive && d <= 0.0) reject(label + " must be positive");
    return d;
}

double finite_value(double d, const std::string &label, NumberRule rule) {
    JValue v;
    v.kind = JKind::Float;
    v.number = d;
    return number_of(v, label, rule);
}

// Python's `x == 1 or x == -1` on a JSON value, and its str() for the IR line.
bool unit_entry(const JValue &v, std::string *text) {
    if (v.kind == JKind::Bool && v.boolean) {
        *text = "True";
        return true;
    }
    if (v.kind == JKind::Int && (v.integer.compare_small(1) == 0 || v.integer.compare_small(-1) == 0)) {
        *text = v.integer.decimal();
        return true;
    }
    if (v.kind == JKind::Float && (v.number == 1.0 || v.number == -1.0)) {
        *text = py_float(v.number);
        return true;
    }
    return false;
}

std::string g17(double v) {
    char buf[40];
    snprintf(buf, sizeof buf, "%.17g", v);
    return buf;
}

struct CompiledNode {
    std::string name;
    const OpRule *op;
    uint32_t left = 0xffffffffu, right = 0xffffffffu;
    double scalar = 0.0;
    int64_t grade = 0;
    int constraint = 0;
    int requires_grad = 0;
    std::vector<double> value;
};

std::vector<double> initial_value(const JValue *spec, size_t blades, const BigInt &seed, const std::string &name) {
    std::vector<double> values(blades, 0.0);
    if (spec != nullptr && spec->kind == JKind::Array) {
        if (spec->items.size() != blades)
            reject("initializer for " + name + " must contain " + std::to_string(blades) + " coefficients");
        for (size_t k = 0; k < blades; ++k)
            values[k] = number_of(*spec->items[k], "initializer " + name + "[" + std::to_string(k) + "]", kFinite);
        return values;
    }
    if (spec == nullptr || spec->kind == JKind::Null || is_string(spec, "zeros")) return values;
    if (is_string(spec, "ones")) return std::vector<double>(blades, 1.0);
    if (spec->kind != JKind::String) reject("invalid initializer for " + name);
    const std::string text = utf8(spec->text);
    std::vector<std::string> parts;
    for (size_t a = 0;;) {
        const size_t b = text.find(':', a);
        parts.push_back(text.substr(a, b == std::string::npos ? std::string::npos : b - a));
        if (b == std::string::npos) break;
        a = b + 1;
    }
    const std::string &kind = parts[0];
    if (kind == "scalar" && parts.size() == 2) {
        values[0] = finite_value(py_float_of(parts[1]), "initializer " + name, kFinite);
        return values;
    }
    if (kind == "basis" && parts.size() == 3) {
        const BigInt index = py_int_of(parts[1]);
        if (index.compare_small(0) < 0 || index.compare_small((int64_t)blades) >= 0)
            reject("basis index for " + name + " is out of range");
        values[index.words.empty() ? 0 : index.words[0]] =
            finite_value(py_float_of(parts[2]), "initializer " + name, kFinite);
        return values;
    }
    if (kind == "random" && parts.size() <= 3) {
        BigInt local = seed;
        double scale = 0.1;
        if (parts.size() >= 2 && !parts[1].empty()) local = py_int_of(parts[1]);
        if (parts.size() == 3) scale = finite_value(py_float_of(parts[2]), "random scale for " + name, kPositive);
        uint32_t code_sum = 0;
        for (unsigned char c : name) code_sum += c;  // names are ASCII
        Mt19937 rng(random_key(local, code_sum));
        for (size_t k = 0; k < blades; ++k) values[k] = -scale + (scale - -scale) * rng.unit();
        return values;
    }
    reject("unsupported initializer '" + text + "' for " + name);
}

bool valid_name(const JValue *v) {
    if (v == nullptr || v->kind != JKind::String || v->text.empty() || v->text.size() > 63) return false;
    for (size_t k = 0; k < v->text.size(); ++k) {
        const char32_t c = v->text[k];
        const bool alpha = (c >= U'A' && c <= U'Z') || (c >= U'a' && c <= U'z') || c == U'_';
        if (!(alpha || (k > 0 && c >= U'0' && c <= U'9'))) return false;
    }
    return true;
}

template <typename T, size_t N>
const T *find_code(const T (&table)[N], const JValue *v) {
    if (v == nullptr || v->kind != JKind::String) return nullptr;
    const std::string s = utf8(v->text);
    for (const T &e : table)
        if (s == e.name) return &e;
    return nullptr;
}

const JValue *section(const JValue &root, const char *key, const char *what) {
    const JValue *v = root.get(key);
    if (v != nullptr && v->kind != JKind::Object) reject(std::string(what) + " must be an object");
    return v;
}

struct Compiled {
    std::string ir;
    std::string summary;
};

Compiled compile_document(const JValue &doc) {
    // -- root
    if (doc.kind != JKind::Object) reject("model root must be an object");
    std::vector<std::string> unknown;
    for (const auto &m : doc.members) {
        const std::string k = utf8(m.first);
        if (std::find_if(std::begin(kRootKeys), std::end(kRootKeys), [&](const char *r) { return k == r; }) ==
            std::end(kRootKeys))
            unknown.push_back(k);
    }
    if (!unknown.empty()) {
        std::sort(unknown.begin(), unknown.end());
        std::string list;
        for (size_t k = 0; k < unknown.size(); ++k) list += (k ? ", " : "") + unknown[k];
        reject("unknown root keys: " + list);
    }
    const JValue *version = doc.get("version");
    const bool version_ok = version != nullptr &&
                            ((version->kind == JKind::Int && version->integer.compare_small(8) == 0) ||
                             (version->kind == JKind::Float && version->number == 8.0));
    if (!version_ok) reject("version must be 8");
    const JValue *dim = doc.get("dimension");
    if (dim == nullptr || dim->kind != JKind::Int || dim->integer.compare_small(1) < 0 ||
        dim->integer.compare_small(6) > 0)
        reject("dimension must be an integer from 1 through 6");
    const unsigned dimension = dim->integer.words[0];
    const JValue *sig = doc.get("signature");
    std::vector<std::string> sig_text;
    bool sig_ok = sig != nullptr && sig->kind == JKind::Array && sig->items.size() == dimension;
    for (size_t k = 0; sig_ok && k < sig->items.size(); ++k) {
        std::string t;
        sig_ok = unit_entry(*sig->items[k], &t);
        sig_text.push_back(t);
    }
    if (!sig_ok) reject("signature must contain exactly dimension entries, each +1 or -1");
    BigInt seed;
    seed.words.push_back(1);
    if (const JValue *s = doc.get("seed")) {
        if (s->kind != JKind::Int || s->integer.negative) reject("seed must be a nonnegative integer");
        seed = s->integer;
    }
    const JValue *nodes = doc.get("nodes");
    if (nodes == nullptr || nodes->kind != JKind::Array || nodes->items.empty())
        reject("nodes must be a nonempty array");
    const JValue *optimizer = section(doc, "optimizer", "optimizer");
    const JValue *training = section(doc, "training", "training");
    const JValue *dataset = section(doc, "dataset", "dataset");

    // -- nodes, in order; each may refer only to earlier ones
    const size_t blades = (size_t)1 << dimension;
    std::vector<CompiledNode> compiled;
    std::map<std::string, uint32_t> index_of;
    for (size_t i = 0; i < nodes->items.size(); ++i) {
        const JValue &raw = *nodes->items[i];
        const std::string at = "node " + std::to_string(i);
        if (raw.kind != JKind::Object) reject(at + " must be an object");
        std::vector<std::string> extra;
        for (const auto &m : raw.members) {
            const std::string k = utf8(m.first);
            if (std::find_if(std::begin(kNodeKeys), std::end(kNodeKeys), [&](const char *r) { return k == r; }) ==
                std::end(kNodeKeys))
                extra.push_back(k);
        }
        if (!extra.empty()) {
            std::sort(extra.begin(), extra.end());
            std::string list;
            for (size_t k = 0; k < extra.size(); ++k) list += (k ? ", " : "") + extra[k];
            reject(at + " has unknown keys: " + list);
        }
        const JValue *name_v = raw.get("name");
        if (!valid_name(name_v)) reject(at + " has an invalid name");
        CompiledNode node;
        node.name = utf8(name_v->text);
        if (index_of.count(node.name)) reject("duplicate node name '" + node.name + "'");
        const JValue *op_v = raw.get("op");
        node.op = find_code(kOps, op_v);
        if (node.op == nullptr) {
            JValue none;
            reject("node " + node.name + " has unsupported op '" + py_str(op_v ? *op_v : none) + "'");
        }
        const std::string self = "node " + node.name;
        const JValue *scalar_v = raw.get("scalar");
        node.scalar = scalar_v ? number_of(*scalar_v, self + " scalar", kFinite) : 0.0;
        if (const JValue *g = raw.get("grade")) {
            if (g->kind != JKind::Int || g->integer.compare_small(0) < 0 ||
                g->integer.compare_small((int64_t)dimension) > 0)
                reject(self + " grade is invalid");
            node.grade = g->integer.words.empty() ? 0 : g->integer.words[0];
        }
        const JValue *c_v = raw.get("constraint");
        const Code *constraint = c_v ? find_code(kConstraints, c_v) : &kConstraints[0];
        if (constraint == nullptr) reject(self + " has invalid constraint");
        node.constraint = constraint->code;
        bool requires_grad = node.op->code == 3;
        if (const JValue *rg = raw.get("requires_grad")) {
            if (rg->kind != JKind::Bool) reject(self + " requires_grad must be boolean");
            requires_grad = rg->boolean;
        }
        node.value = initial_value(raw.get("init"), blades, seed, node.name);
        auto present = [&](const char *k) {
            const JValue *v = raw.get(k);
            return v != nullptr && v->kind != JKind::Null;
        };
        if (node.op->arity == kLeaf) {
            if (present("inputs") || present("input")) reject("leaf node " + node.name + " cannot have inputs");
            if (node.op->code != 3 && node.constraint != 0)
                reject("constraint is valid only on parameter node " + node.name);
        } else if (node.op->arity == kOneInput) {
            const JValue *in = raw.get("input");
            if (in == nullptr || in->kind != JKind::String || !index_of.count(utf8(in->text)))
                reject(self + " must reference one earlier input");
            node.left = index_of[utf8(in->text)];
        } else {
            const JValue *ins = raw.get("inputs");
            bool two = ins != nullptr && ins->kind == JKind::Array && ins->items.size() == 2;
            for (size_t k = 0; two && k < 2; ++k) two = ins->items[k]->kind == JKind::String;
            if (!two) reject(self + " must have two inputs");
            for (size_t k = 0; k < 2; ++k)
                if (!index_of.count(utf8(ins->items[k]->text)))
                    reject(self + " references an unknown or forward input");
            node.left = index_of[utf8(ins->items[0]->text)];
            node.right = index_of[utf8(ins->items[1]->text)];
        }
        if (node.op->arity != kLeaf) {
            node.value.assign(blades, 0.0);
            node.constraint = 0;
            requires_grad = false;
        }
        node.requires_grad = requires_grad ? 1 : 0;
        if (node.op->code == 16 && node.scalar == 0.0) node.scalar = 1e-12;
        if (node.op->code != 10 && raw.has("grade")) reject("grade is only valid for grade_project node " + node.name);
        if (node.op->code != 7 && node.op->code != 16 && raw.has("scalar"))
            reject("scalar is not valid for node " + node.name);
        index_of[node.name] = (uint32_t)i;
        compiled.push_back(std::move(node));
    }

    // -- graph ends and state bindings
    auto named = [&](const char *key, const char *message) -> uint32_t {
        const JValue *v = doc.get(key);
        if (v == nullptr || v->kind != JKind::String || !index_of.count(utf8(v->text))) reject(message);
        return index_of[utf8(v->text)];
    };
    const uint32_t loss = named("loss", "loss must name an existing node");
    const uint32_t output = named("output", "output must name an existing node");
    std::vector<std::pair<uint32_t, uint32_t>> bindings;
    if (const JValue *su = doc.get("state_updates")) {
        if (su->kind != JKind::Object) reject("state_updates must be an object");
        std::vector<std::pair<std::u32string, const JValue *>> sorted;
        for (const auto &m : su->members) sorted.emplace_back(m.first, m.second.get());
        std::sort(sorted.begin(), sorted.end(), [](const auto &a, const auto &b) { return a.first < b.first; });
        for (const auto &e : sorted) {
            const std::string state = utf8(e.first);
            if (!index_of.count(state) || e.second->kind != JKind::String || !index_of.count(utf8(e.second->text)))
                reject("state update references an unknown node");
            if (compiled[index_of[state]].op->code != 5) reject("state update key '" + state + "' is not a state");
            bindings.emplace_back(index_of[state], index_of[utf8(e.second->text)]);
        }
    }
    std::vector<std::string> unbound;
    size_t states = 0;
    for (size_t i = 0; i < compiled.size(); ++i) {
        if (compiled[i].op->code != 5) continue;
        ++states;
        if (std::none_of(bindings.begin(), bindings.end(), [&](const auto &b) { return b.first == i; }))
            unbound.push_back(compiled[i].name);
    }
    if (!unbound.empty()) {
        std::string list;
        for (size_t k = 0; k < unbound.size(); ++k) list += (k ? ", " : "") + unbound[k];
        reject("every state requires an update binding: " + list);
    }

    // -- optimizer, training, dataset
    const JValue *type = optimizer ? optimizer->get("type") : nullptr;
    const Code *opt = type ? find_code(kOptimizers, type) : &kOptimizers[1];
    if (opt == nullptr) reject("optimizer.type must be sgd or adam");
    double hyper[4];
    for (size_t k = 0; k < 4; ++k) {
        const NumberField &f = kOptimizerNumbers[k];
        const JValue *v = optimizer ? optimizer->get(f.key) : nullptr;
        hyper[k] = v ? number_of(*v, f.label, f.rule) : f.fallback;
    }
    if (!(hyper[1] >= 0.0 && hyper[1] < 1.0) || !(hyper[2] >= 0.0 && hyper[2] < 1.0))
        reject("optimizer beta values must be in [0,1)");
    std::string counts[2];
    for (size_t k = 0; k < 2; ++k) {
        const JValue *v = training ? training->get(kTrainingCounts[k].key) : nullptr;
        if (v == nullptr) {
            counts[k] = "1";
            continue;
        }
        if (v->kind != JKind::Int || v->integer.compare_small(0) <= 0)
            reject(std::string(kTrainingCounts[k].label) + " must be a positive integer");
        counts[k] = v->integer.decimal();
    }
    bool reset_each_epoch = true;
    if (const JValue *v = training ? training->get("reset_state_each_epoch") : nullptr) {
        if (v->kind != JKind::Bool) reject("training.reset_state_each_epoch must be boolean");
        reset_each_epoch = v->boolean;
    }
    bool reset_column = states > 0;
    if (const JValue *v = dataset ? dataset->get("reset_column") : nullptr) {
        if (v->kind != JKind::Bool) reject("dataset.reset_column must be boolean");
        reset_column = v->boolean;
    }

    // -- IR text
    std::string ir = "geo_model_ir=8\ndimension=" + std::to_string(dimension) + "\nsignature=";
    for (size_t k = 0; k < sig_text.size(); ++k) ir += (k ? "," : "") + sig_text[k];
    ir += "\noptimizer=" + std::to_string(opt->code);
    const char *hyper_keys[4] = {"learning_rate", "beta1", "beta2", "epsilon"};
    for (size_t k = 0; k < 4; ++k) ir += std::string("\n") + hyper_keys[k] + "=" + g17(hyper[k]);
    ir += "\nepochs=" + counts[0] + "\nbatch_size=" + counts[1];
    ir += "\nreset_state_each_epoch=" + std::to_string((int)reset_each_epoch);
    ir += "\nreset_column=" + std::to_string((int)reset_column);
    ir += "\nnode_count=" + std::to_string(compiled.size());
    ir += "\nloss=" + std::to_string(loss) + "\noutput=" + std::to_string(output) + "\n";
    size_t counts_of[4] = {0, 0, 0, 0};  // parameters, inputs, targets
    for (size_t i = 0; i < compiled.size(); ++i) {
        const CompiledNode &n = compiled[i];
        ir += "node=" + std::to_string(i) + "," + std::to_string(n.op->code) + "," + n.name + "," +
              std::to_string(n.left) + "," + std::to_string(n.right) + "," + g17(n.scalar) + "," +
              std::to_string(n.grade) + "," + std::to_string(n.constraint) + "," + std::to_string(n.requires_grad) +
              "\nvalue=";
        for (size_t k = 0; k < n.value.size(); ++k) ir += (k ? "," : "") + g17(n.value[k]);
        ir += "\n";
        if (n.op->code == 3) ++counts_of[0];
        if (n.op->code == 1) ++counts_of[1];
        if (n.op->code == 2) ++counts_of[2];
    }
    for (const auto &b : bindings) ir += "state_update=" + std::to_string(b.first) + "," + std::to_string(b.second) + "\n";
    ir += "end=1\n";
    const std::string summary = "nodes=" + std::to_string(compiled.size()) +
                                " parameters=" + std::to_string(counts_of[0]) +
                                " inputs=" + std::to_string(counts_of[1]) + " targets=" + std::to_string(counts_of[2]) +
                                " states=" + std::to_string(states) + " blade_count=" + std::to_string(blades) +
                                " batch_size=" + counts[1];
    return Compiled{ir, summary};
}

bool read_file(const char *path, std::string *out, std::string *error) {
    FILE *f = fopen(path, "rb");
    if (f == nullptr) {
        const int e = errno;
        *error = "[Errno " + std::to_string(e) + "] " + strerror(e) + ": " + py_repr_str(widen(path));
        return false;
    }
    char buf[65536];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) out->append(buf, n);
    fclose(f);
    return true;
}

// Writes `text` to a temporary file beside `path`, flushes it to disk and renames it over `path`.
bool write_atomically(const char *path, const std::string &text, std::string *error) {
    std::string tmpl = std::string(path) + ".XXXXXX";
    std::vector<char> name(tmpl.begin(), tmpl.end());
    name.push_back('\0');
    const int fd = mkstemp(name.data());
    if (fd < 0) {
        *error = std::string("[Errno ") + std::to_string(errno) + "] " + strerror(errno) + ": " +
                 py_repr_str(widen(path));
        return false;
    }
    bool ok = write(fd, text.data(), text.size()) == (ssize_t)text.size() && fsync(fd) == 0;
    ok = close(fd) == 0 && ok;
    if (ok && rename(name.data(), path) != 0) ok = false;
    if (!ok) {
        *error = std::string("[Errno ") + std::to_string(errno) + "] " + strerror(errno) + ": " +
                 py_repr_str(widen(path));
        unlink(name.data());
    }
    return ok;
}

void copy_out(const std::string &s, char *buf, size_t cap) {
    if (buf == nullptr || cap == 0) return;
    const size_t n = std::min(s.size(), cap - 1);
    memcpy(buf, s.data(), n);
    buf[n] = '\0';
}

}  // namespace

extern "C" int geo_b200_model_compile_text(const char *json_text, size_t json_length, char **ir_text,
                                           char *summary, size_t summary_capacity, char *error,
                                           size_t error_capacity) {
    if (ir_text != nullptr) *ir_text = nullptr;
    try {
        if (json_text == nullptr) throw Failure{"no model text"};
        const JPtr doc = Reader(decode_text(std::string(json_text, json_length))).document();
        const Compiled c = compile_document(*doc);
        if (ir_text != nullptr) {
            *ir_text = static_cast<char *>(malloc(c.ir.size() + 1));
            if (*ir_text == nullptr) throw Failure{"out of memory"};
            memcpy(*ir_text, c.ir.c_str(), c.ir.size() + 1);
        }
        copy_out(c.summary, summary, summary_capacity);
        copy_out("", error, error_capacity);
        return 1;
    } catch (const Failure &f) {
        copy_out(f.message, error, error_capacity);
        return 0;
    }
}

extern "C" void geo_b200_model_free_text(char *text) { free(text); }

extern "C" int geo_b200_model_compile(const char *model_path, const char *ir_path) {
    std::string text, error;
    char summary[512], message[1024];
    char *ir = nullptr;
    if (model_path == nullptr || !read_file(model_path, &text, &error)) {
        fprintf(stderr, "geo_model: %s\n", error.c_str());
        return 0;
    }
    if (!geo_b200_model_compile_text(text.data(), text.size(), ir_path ? &ir : nullptr, summary, sizeof summary,
                                     message, sizeof message)) {
        fprintf(stderr, "geo_model: %s\n", message);
        return 0;
    }
    if (ir_path != nullptr) {
        const bool ok = write_atomically(ir_path, ir, &error);
        geo_b200_model_free_text(ir);
        if (!ok) {
            fprintf(stderr, "geo_model: %s\n", error.c_str());
            return 0;
        }
        printf("GEO_MODEL_COMPILE: PASS output=%s %s\n", ir_path, summary);
    } else {
        printf("GEO_MODEL_VALIDATE: PASS %s\n", summary);
    }
    fflush(stdout);
    return 1;
}
