// tokenizer.cpp -- host byte-level BPE tokenizer behind the C-ABI
// (b2_tokenizer_*, include/b2engine.h).  Replaces engine::BPETokenizer
// (src/tokenizer/bpe.h:17-58, bpe.cpp) and widens it from the Qwen2 vocabulary
// to the Llama-3 and GPT-2 ones: everything a HF tokenizer.json of the
// byte-level BPE family says is read from the file --
//
//   normalizer      null or NFC (Qwen2 ships NFC; the reference skips it)
//   pre_tokenizer   Split on the Qwen2 pattern (bpe.cpp:170, one digit per
//                   piece) or the Llama-3 pattern (runs of up to three
//                   digits), then ByteLevel; or ByteLevel with its own
//                   GPT-2 pattern
//   model           BPE: vocab, merges ("a b" strings or [a, b] pairs),
//                   ignore_merges (Llama-3: a piece that is itself a vocab
//                   entry is one token)
//   added_tokens    split out of the text before normalisation (or after
//                   it, for tokens marked normalized), longest match at the
//                   leftmost position; special ones only when asked
//                   (bpe.cpp:394-431), lstrip / rstrip / single_word honoured
//   post_processor  TemplateProcessing (Llama-3's <|begin_of_text|>) applied
//                   when the caller asks for special tokens
//
// Text is handled as bytes throughout: pieces are byte ranges of the input,
// vocab entries are kept as the bytes they stand for, and merges are keyed on
// token-id pairs, so no string is re-encoded on the way.  Bytes that are not
// valid UTF-8 cannot reach the HF library; here each such byte is a character
// of its own outside every class and passes through to its byte token, so
// decode(encode(x)) == x for any byte string.
//
// Merging follows the BPE definition the reference applies (bpe.cpp:322-358,
// lowest-ranked adjacent pair first, leftmost among equals) with a heap over
// a linked list of symbols instead of rescanning the word per merge.
#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/b2engine.h"

// records the failure text b2_last_error() returns (model.cu)
void b2_record_error(const char* msg);

namespace {

struct CpRange { uint32_t lo, hi; };
struct CccRange { uint32_t lo, hi; uint8_t ccc; };
struct DecompEntry { uint32_t cp; uint32_t off; uint8_t len; };
struct ComposePair { uint32_t a, b, c; };
#include "unicode_tables.inc"

template <size_t N>
bool in_ranges(const CpRange (&r)[N], uint32_t cp) {
    size_t lo = 0, hi = N;
    while (lo < hi) {
        size_t mid = (lo + hi) / 2;
        if (cp < r[mid].lo) hi = mid;
        else if (cp > r[mid].hi) lo = mid + 1;
        else return true;
    }
    return false;
}

// Code points above 0x10FFFF stand for single bytes that are not valid UTF-8.
constexpr uint32_t kRawByte = 0x110000;

enum CharClass : uint8_t { C_OTHER = 0, C_LETTER = 1, C_NUMBER = 2, C_SPACE = 3 };

inline uint8_t char_class(uint32_t cp) {
    if (cp < 0x80) {
        if ((cp | 0x20) >= 'a' && (cp | 0x20) <= 'z') return C_LETTER;
        if (cp >= '0' && cp <= '9') return C_NUMBER;
        if (cp == ' ' || (cp >= 0x09 && cp <= 0x0D)) return C_SPACE;
        return C_OTHER;
    }
    if (cp >= kRawByte) return C_OTHER;
    if (in_ranges(kLetterRanges, cp)) return C_LETTER;
    if (in_ranges(kNumberRanges, cp)) return C_NUMBER;
    if (in_ranges(kSpaceRanges, cp)) return C_SPACE;
    return C_OTHER;
}

// One UTF-8 character at s[0..n): its code point and length.  Overlong forms,
// surrogates, values above 0x10FFFF and truncated or stray bytes decode as
// kRawByte + byte, length 1.
inline uint32_t next_cp(const uint8_t* s, size_t n, size_t* len) {
    uint8_t c = s[0];
    if (c < 0x80) { *len = 1; return c; }
    int need; uint32_t cp, min;
    if ((c & 0xE0) == 0xC0) { need = 1; cp = c & 0x1F; min = 0x80; }
    else if ((c & 0xF0) == 0xE0) { need = 2; cp = c & 0x0F; min = 0x800; }
    else if ((c & 0xF8) == 0xF0) { need = 3; cp = c & 0x07; min = 0x10000; }
    else { *len = 1; return kRawByte + c; }
    if ((size_t)need >= n) { *len = 1; return kRawByte + c; }
    for (int k = 1; k <= need; ++k) {
        if ((s[k] & 0xC0) != 0x80) { *len = 1; return kRawByte + c; }
        cp = (cp << 6) | (s[k] & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) { *len = 1; return kRawByte + c; }
    *len = (size_t)need + 1;
    return cp;
}

inline void put_cp(std::string& out, uint32_t cp) {
    if (cp >= kRawByte) { out.push_back((char)(cp - kRawByte)); return; }
    if (cp < 0x80) out.push_back((char)cp);
    else if (cp < 0x800) { out.push_back((char)(0xC0 | (cp >> 6))); out.push_back((char)(0x80 | (cp & 0x3F))); }
    else if (cp < 0x10000) {
        out.push_back((char)(0xE0 | (cp >> 12)));
        out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
        out.push_back((char)(0x80 | (cp & 0x3F)));
    } else {
        out.push_back((char)(0xF0 | (cp >> 18)));
        out.push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
        out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
        out.push_back((char)(0x80 | (cp & 0x3F)));
    }
}

// ---------------------------------------------------------------------------
// NFC (canonical decomposition, canonical ordering, canonical composition;
// Hangul syllables by arithmetic) over the tables the generator read off the
// HF library's normaliser.

constexpr uint32_t kSBase = 0xAC00, kLBase = 0x1100, kVBase = 0x1161, kTBase = 0x11A7;
constexpr uint32_t kLCount = 19, kVCount = 21, kTCount = 28, kNCount = kVCount * kTCount, kSCount = kLCount * kNCount;

inline uint8_t ccc_of(uint32_t cp) {
    if (cp < 0x300 || cp >= kRawByte) return 0;
    size_t lo = 0, hi = sizeof(kCccRanges) / sizeof(kCccRanges[0]);
    while (lo < hi) {
        size_t mid = (lo + hi) / 2;
        if (cp < kCccRanges[mid].lo) hi = mid;
        else if (cp > kCccRanges[mid].hi) lo = mid + 1;
        else return kCccRanges[mid].ccc;
    }
    return 0;
}

void decompose(uint32_t cp, std::vector<uint32_t>& out) {
    if (cp >= kSBase && cp < kSBase + kSCount) {
        uint32_t s = cp - kSBase;
        out.push_back(kLBase + s / kNCount);
        out.push_back(kVBase + (s % kNCount) / kTCount);
        if (s % kTCount) out.push_back(kTBase + s % kTCount);
        return;
    }
    if (cp >= 0xC0 && cp < kRawByte) {
        const DecompEntry* b = kDecomp;
        const DecompEntry* e = kDecomp + sizeof(kDecomp) / sizeof(kDecomp[0]);
        const DecompEntry* it = std::lower_bound(b, e, cp, [](const DecompEntry& d, uint32_t v) { return d.cp < v; });
        if (it != e && it->cp == cp) {
            out.insert(out.end(), kDecompData + it->off, kDecompData + it->off + it->len);
            return;
        }
    }
    out.push_back(cp);
}

inline uint32_t compose_pair(uint32_t a, uint32_t b) {
    if (a >= kLBase && a < kLBase + kLCount && b >= kVBase && b < kVBase + kVCount)
        return kSBase + ((a - kLBase) * kVCount + (b - kVBase)) * kTCount;
    if (a >= kSBase && a < kSBase + kSCount && (a - kSBase) % kTCount == 0 && b > kTBase && b < kTBase + kTCount)
        return a + (b - kTBase);
    const ComposePair* bg = kCompose;
    const ComposePair* e = kCompose + sizeof(kCompose) / sizeof(kCompose[0]);
    const ComposePair* it = std::lower_bound(bg, e, std::make_pair(a, b), [](const ComposePair& p, std::pair<uint32_t, uint32_t> v) {
        return p.a < v.first || (p.a == v.first && p.b < v.second);
    });
    return (it != e && it->a == a && it->b == b) ? it->c : 0;
}

// Full NFC of s[0..n), appended to out.
void nfc_full(const uint8_t* s, size_t n, std::string& out) {
    std::vector<uint32_t> cps;
    cps.reserve(n);
    for (size_t i = 0; i < n;) {
        size_t len;
        uint32_t cp = next_cp(s + i, n - i, &len);
        decompose(cp, cps);
        i += len;
    }
    // canonical ordering: stable sort of each run of non-starters by class
    for (size_t i = 0; i < cps.size();) {
        if (ccc_of(cps[i]) == 0) { ++i; continue; }
        size_t j = i;
        while (j < cps.size() && ccc_of(cps[j]) != 0) ++j;
        if (j - i > 1)
            std::stable_sort(cps.begin() + i, cps.begin() + j, [](uint32_t x, uint32_t y) { return ccc_of(x) < ccc_of(y); });
        i = j;
    }
    // canonical composition
    std::vector<uint32_t> res;
    res.reserve(cps.size());
    long starter = -1;
    int last_ccc = -1;   // class of the last character kept after the starter (-1: none)
    for (uint32_t cp : cps) {
        int c = ccc_of(cp);
        if (starter >= 0 && (last_ccc == -1 || (last_ccc < c))) {
            uint32_t comp = compose_pair(res[starter], cp);
            if (comp) { res[starter] = comp; continue; }
        }
        if (c == 0) { starter = (long)res.size(); last_ccc = -1; }
        else last_ccc = c;
        res.push_back(cp);
    }
    for (uint32_t cp : res) put_cp(out, cp);
}

// Code points NFC may change or join to a neighbour: non-starters, the second
// characters of composition pairs (Hangul vowel and trailing jamo included),
// and characters whose own NFC differs from them (singletons, excluded and
// non-starter decompositions).  Anything else is a boundary: nothing before
// it interacts with anything after it except through characters in this set.
struct NfcUnstable {
    std::vector<uint64_t> bits = std::vector<uint64_t>((0x110000 + 63) / 64, 0);
    void set(uint32_t cp) { bits[cp >> 6] |= 1ull << (cp & 63); }
    bool get(uint32_t cp) const { return cp < 0x110000 && ((bits[cp >> 6] >> (cp & 63)) & 1); }
    NfcUnstable() {
        for (const CccRange& r : kCccRanges)
            for (uint32_t c = r.lo; c <= r.hi; ++c) set(c);
        for (const ComposePair& p : kCompose) set(p.b);
        for (uint32_t c = kVBase; c < kVBase + kVCount; ++c) set(c);
        for (uint32_t c = kTBase + 1; c < kTBase + kTCount; ++c) set(c);
        for (const DecompEntry& d : kDecomp) {
            std::string one, back;
            put_cp(one, d.cp);
            nfc_full((const uint8_t*)one.data(), one.size(), back);
            if (back != one) set(d.cp);
        }
    }
};

// NFC of s[0..n) into out: runs of characters outside NfcUnstable are copied;
// each run of unstable ones goes through the full algorithm together with the
// stable character before it (a starter it may compose with).  Text whose
// code points are all below U+0300 is NFC already and is copied whole.
void nfc(const uint8_t* s, size_t n, std::string& out) {
    bool simple = true;
    for (size_t i = 0; i < n && simple; ++i)
        if (s[i] >= 0xCC) simple = false;   // lead bytes of U+0300 and above
    if (simple) { out.append((const char*)s, n); return; }
    static const NfcUnstable unstable;
    size_t copied = 0, last_stable = 0;
    bool have_stable = false;
    for (size_t i = 0; i < n;) {
        size_t len;
        uint32_t cp = next_cp(s + i, n - i, &len);
        if (!unstable.get(cp)) { last_stable = i; have_stable = true; i += len; continue; }
        size_t ws = have_stable && last_stable >= copied ? last_stable : copied, j = i + len;
        while (j < n) {
            size_t l2;
            if (!unstable.get(next_cp(s + j, n - j, &l2))) break;
            j += l2;
        }
        out.append((const char*)s + copied, ws - copied);
        nfc_full(s + ws, j - ws, out);
        copied = i = j;
        have_stable = false;
    }
    out.append((const char*)s + copied, n - copied);
}

// ---------------------------------------------------------------------------
// Pre-tokenizer: the three byte-level BPE split patterns, matched by hand.
//   QWEN2  (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}|
//          ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+
//   LLAMA3 the same with \p{N}{1,3}
//   GPT2   's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+
// Every character starts a match under each pattern, so the pieces tile the
// text.

enum PreKind { PRE_QWEN2 = B2_PRE_QWEN2, PRE_LLAMA3 = B2_PRE_LLAMA3, PRE_GPT2 = B2_PRE_GPT2 };

const char* kQwen2Pattern =
    "(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}| ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*|\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+";
const char* kLlama3Pattern =
    "(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}{1,3}| ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*|\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+";

struct Ch { uint32_t cp; uint32_t off; uint8_t cls; };

inline bool is_crlf(uint32_t cp) { return cp == '\r' || cp == '\n'; }

// Contraction after an apostrophe at c[i]: characters matched (0: none).
// `fold`: the case-insensitive form, where s also matches U+017F (long s).
size_t contraction(const Ch* c, size_t i, size_t n, bool fold) {
    if (c[i].cp != '\'' || i + 1 >= n) return 0;
    auto eq = [fold](uint32_t cp, char lower) {
        if (cp == (uint32_t)lower) return true;
        if (!fold) return false;
        if (cp == (uint32_t)(lower - 32)) return true;
        return lower == 's' && cp == 0x17F;
    };
    uint32_t a = c[i + 1].cp;
    if (eq(a, 's') || eq(a, 't')) return 2;
    if (i + 2 < n) {
        uint32_t b = c[i + 2].cp;
        if ((eq(a, 'r') && eq(b, 'e')) || (eq(a, 'v') && eq(b, 'e'))) return 3;
    }
    if (eq(a, 'm')) return 2;
    if (i + 2 < n && eq(a, 'l') && eq(c[i + 2].cp, 'l')) return 3;
    if (eq(a, 'd')) return 2;
    return 0;
}

size_t run_of(const Ch* c, size_t j, size_t n, uint8_t cls) {
    while (j < n && c[j].cls == cls) ++j;
    return j;
}

// Length in characters of the match that starts at c[i] (always >= 1).
size_t match_piece(const Ch* c, size_t i, size_t n, int kind) {
    const Ch& c0 = c[i];
    if (kind == PRE_GPT2) {
        if (size_t k = contraction(c, i, n, false)) return k;
        size_t s = (c0.cp == ' ' && i + 1 < n) ? i + 1 : i;
        for (uint8_t cls : {C_LETTER, C_NUMBER, C_OTHER}) {
            if (c[s].cls == cls) return run_of(c, s + 1, n, cls) - i;
            if (s != i && c0.cls == cls) return run_of(c, i + 1, n, cls) - i;
        }
    } else {
        if (size_t k = contraction(c, i, n, true)) return k;
        // [^\r\n\p{L}\p{N}]?\p{L}+
        if (c0.cls == C_LETTER) return run_of(c, i + 1, n, C_LETTER) - i;
        if (!is_crlf(c0.cp) && c0.cls != C_NUMBER && i + 1 < n && c[i + 1].cls == C_LETTER)
            return run_of(c, i + 2, n, C_LETTER) - i;
        // \p{N} or \p{N}{1,3}
        if (c0.cls == C_NUMBER) {
            size_t lim = kind == PRE_LLAMA3 ? 3 : 1, j = i + 1;
            while (j < n && j - i < lim && c[j].cls == C_NUMBER) ++j;
            return j - i;
        }
        //  ?[^\s\p{L}\p{N}]+[\r\n]*
        size_t s = (c0.cp == ' ' && i + 1 < n && c[i + 1].cls == C_OTHER) ? i + 1 : i;
        if (c[s].cls == C_OTHER) {
            size_t j = run_of(c, s + 1, n, C_OTHER);
            while (j < n && is_crlf(c[j].cp)) ++j;
            return j - i;
        }
        // \s*[\r\n]+ : through the last CR/LF of the whitespace run
        size_t j = run_of(c, i, n, C_SPACE), last = 0;
        for (size_t k = i; k < j; ++k)
            if (is_crlf(c[k].cp)) last = k + 1;
        if (last) return last - i;
    }
    // \s+(?!\S) then \s+
    size_t j = run_of(c, i, n, C_SPACE);
    if (j == i) return 1;   // not reached: every class is covered above
    if (j == n || j - i == 1) return j - i;
    return j - i - 1;
}

// ---------------------------------------------------------------------------
// Minimal JSON reader (what tokenizer.json needs: objects, arrays, strings
// with escapes, numbers, literals).

struct JVal {
    enum T : uint8_t { NUL, BOOL, NUM, STR, ARR, OBJ } t = NUL;
    bool b = false;
    double num = 0;
    std::string s;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal* get(const char* k) const {
        if (t != OBJ) return nullptr;
        for (auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
    bool is_true(const char* k) const { const JVal* v = get(k); return v && v->t == BOOL && v->b; }
    const std::string* str(const char* k) const { const JVal* v = get(k); return v && v->t == STR ? &v->s : nullptr; }
};

struct JParser {
    const char* p;
    const char* e;
    std::string err;
    void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
    bool fail(const char* m) { if (err.empty()) err = m; return false; }
    bool hex4(uint32_t& v) {
        if (e - p < 4) return fail("truncated \\u escape");
        v = 0;
        for (int k = 0; k < 4; ++k) {
            char ch = *p++;
            v <<= 4;
            if (ch >= '0' && ch <= '9') v |= ch - '0';
            else if (ch >= 'a' && ch <= 'f') v |= ch - 'a' + 10;
            else if (ch >= 'A' && ch <= 'F') v |= ch - 'A' + 10;
            else return fail("bad \\u escape");
        }
        return true;
    }
    bool string(std::string& out) {
        if (p >= e || *p != '"') return fail("expected string");
        ++p;
        while (p < e && *p != '"') {
            if (*p != '\\') {
                const char* q = p;
                while (q < e && *q != '"' && *q != '\\') ++q;
                out.append(p, q - p);
                p = q;
                continue;
            }
            if (++p >= e) return fail("truncated escape");
            char ch = *p++;
            switch (ch) {
            case '"': out.push_back('"'); break;
            case '\\': out.push_back('\\'); break;
            case '/': out.push_back('/'); break;
            case 'b': out.push_back('\b'); break;
            case 'f': out.push_back('\f'); break;
            case 'n': out.push_back('\n'); break;
            case 'r': out.push_back('\r'); break;
            case 't': out.push_back('\t'); break;
            case 'u': {
                uint32_t v;
                if (!hex4(v)) return false;
                if (v >= 0xD800 && v < 0xDC00 && e - p >= 6 && p[0] == '\\' && p[1] == 'u') {
                    const char* save = p;
                    p += 2;
                    uint32_t lo;
                    if (!hex4(lo)) return false;
                    if (lo >= 0xDC00 && lo < 0xE000) v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
                    else p = save;
                }
                put_cp(out, v);
                break;
            }
            default: return fail("bad escape");
            }
        }
        if (p >= e) return fail("unterminated string");
        ++p;
        return true;
    }
    bool value(JVal& v, int depth) {
        if (depth > 64) return fail("nesting too deep");
        ws();
        if (p >= e) return fail("unexpected end");
        char ch = *p;
        if (ch == '{') {
            v.t = JVal::OBJ;
            ++p; ws();
            if (p < e && *p == '}') { ++p; return true; }
            for (;;) {
                ws();
                v.obj.emplace_back();
                if (!string(v.obj.back().first)) return false;
                ws();
                if (p >= e || *p != ':') return fail("expected ':'");
                ++p;
                if (!value(v.obj.back().second, depth + 1)) return false;
                ws();
                if (p < e && *p == ',') { ++p; continue; }
                if (p < e && *p == '}') { ++p; return true; }
                return fail("expected ',' or '}'");
            }
        }
        if (ch == '[') {
            v.t = JVal::ARR;
            ++p; ws();
            if (p < e && *p == ']') { ++p; return true; }
            for (;;) {
                v.arr.emplace_back();
                if (!value(v.arr.back(), depth + 1)) return false;
                ws();
                if (p < e && *p == ',') { ++p; continue; }
                if (p < e && *p == ']') { ++p; return true; }
                return fail("expected ',' or ']'");
            }
        }
        if (ch == '"') { v.t = JVal::STR; return string(v.s); }
        if (e - p >= 4 && !memcmp(p, "null", 4)) { p += 4; v.t = JVal::NUL; return true; }
        if (e - p >= 4 && !memcmp(p, "true", 4)) { p += 4; v.t = JVal::BOOL; v.b = true; return true; }
        if (e - p >= 5 && !memcmp(p, "false", 5)) { p += 5; v.t = JVal::BOOL; v.b = false; return true; }
        if (ch == '-' || (ch >= '0' && ch <= '9')) {
            char buf[64];
            size_t k = 0;
            while (p < e && k < sizeof(buf) - 1 && (strchr("+-.eE", *p) || (*p >= '0' && *p <= '9'))) buf[k++] = *p++;
            buf[k] = 0;
            char* end;
            v.t = JVal::NUM;
            v.num = strtod(buf, &end);
            if (end != buf + k) return fail("bad number");
            return true;
        }
        return fail("unexpected character");
    }
};

// ---------------------------------------------------------------------------
// GPT-2 byte alphabet: printable bytes stand for themselves, the other 68
// map in byte order onto U+0100..U+0143.

struct ByteAlphabet {
    int16_t to_byte[0x144];
    ByteAlphabet() {
        int n = 0;
        for (int cp = 0; cp < 0x144; ++cp) to_byte[cp] = -1;
        for (int b = 0; b < 256; ++b) {
            bool printable = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE);
            if (printable) to_byte[b] = (int16_t)b;
            else to_byte[0x100 + n++] = (int16_t)b;
        }
    }
};
const ByteAlphabet kAlphabet;

// The bytes a token string stands for under the byte-level decoder: its
// characters mapped through the alphabet if every one of them is in it,
// otherwise the string's own UTF-8 bytes (`mapped` false).
std::string token_bytes(const std::string& tok, bool* mapped) {
    std::string out;
    out.reserve(tok.size());
    const uint8_t* s = (const uint8_t*)tok.data();
    for (size_t i = 0; i < tok.size();) {
        size_t len;
        uint32_t cp = next_cp(s + i, tok.size() - i, &len);
        if (cp >= 0x144 || kAlphabet.to_byte[cp] < 0) { *mapped = false; return tok; }
        out.push_back((char)kAlphabet.to_byte[cp]);
        i += len;
    }
    *mapped = true;
    return out;
}

// ---------------------------------------------------------------------------

struct AddedToken {
    std::string content;
    int32_t id;
    bool special, normalized, lstrip, rstrip, single_word;
};

// Word characters for single_word added tokens (the library's own set).
inline bool is_word_cp(uint32_t cp) { return cp < kRawByte && in_ranges(kWordRanges, cp); }

// Trie over added-token contents for leftmost-longest matching.
struct Trie {
    struct Node { std::vector<std::pair<uint8_t, int32_t>> next; int32_t token = -1; };
    std::vector<Node> nodes{1};
    void add(const std::string& s, int32_t idx) {
        int32_t cur = 0;
        for (uint8_t ch : s) {
            int32_t nx = -1;
            for (auto& e : nodes[cur].next)
                if (e.first == ch) { nx = e.second; break; }
            if (nx < 0) {
                nx = (int32_t)nodes.size();
                nodes[cur].next.emplace_back(ch, nx);
                nodes.emplace_back();
            }
            cur = nx;
        }
        nodes[cur].token = idx;
    }
    // longest token starting at s[0..n): its index, or -1
    int32_t longest(const uint8_t* s, size_t n, size_t* len) const {
        int32_t cur = 0, best = -1;
        for (size_t k = 0; k < n; ++k) {
            int32_t nx = -1;
            for (auto& e : nodes[cur].next)
                if (e.first == s[k]) { nx = e.second; break; }
            if (nx < 0) break;
            cur = nx;
            if (nodes[cur].token >= 0) { best = nodes[cur].token; *len = k + 1; }
        }
        return best;
    }
    bool empty() const { return nodes[0].next.empty(); }
};

struct PairHash {
    size_t operator()(uint64_t k) const { return (size_t)(k * 0x9E3779B97F4A7C15ull >> 17); }
};

}  // namespace

struct b2_tokenizer {
    int pre = PRE_QWEN2;
    bool use_nfc = false;
    bool ignore_merges = false;
    std::unordered_map<std::string, int32_t> vocab;              // byte form -> id
    std::unordered_map<uint64_t, std::pair<int32_t, int32_t>, PairHash> merges;   // (a,b) -> (rank, merged id)
    std::vector<std::string> id_bytes;                           // id -> bytes it decodes to
    std::vector<uint8_t> id_special;                             // id -> 1 if a special added token
    std::vector<uint8_t> id_valid;
    int32_t byte_id[256];
    std::vector<AddedToken> added;
    Trie raw_trie, norm_trie;                                    // normalized == false / true
    std::vector<int32_t> prefix_ids, suffix_ids;                 // post-processor template
    bool has_template = false;
    size_t vocab_strings = 0;
    int chat = B2_CHAT_NONE;
    int32_t bos = -1, eos = -1;
    std::vector<int32_t> stop;
    std::unordered_map<std::string, int32_t> added_by_content;
};

namespace {

int tok_fail(int code, const std::string& msg) {
    b2_record_error(msg.c_str());
    return code;
}

// Piece of normalised text -> token ids (HF BPE::tokenize with merge_all).
struct BpeSym { int32_t id, prev, next; uint32_t len; };
struct BpeCand { int32_t rank, pos, id; };

void bpe_piece(const b2_tokenizer& t, const uint8_t* s, size_t n, std::vector<int32_t>& out) {
    if (n == 0) return;
    if (n == 1) {  // a single byte is its byte token (or nothing)
        if (t.byte_id[s[0]] >= 0) out.push_back(t.byte_id[s[0]]);
        return;
    }
    if (t.ignore_merges) {
        auto it = t.vocab.find(std::string((const char*)s, n));
        if (it != t.vocab.end()) { out.push_back(it->second); return; }
    }
    // scratch reused across pieces on this thread (encode runs many short pieces)
    thread_local std::vector<BpeSym> syms;
    thread_local std::vector<BpeCand> q;
    using Sym = BpeSym;
    using Cand = BpeCand;
    if (syms.size() < n) syms.resize(n);
    Sym* sy = syms.data();
    int32_t m = 0;
    for (size_t i = 0; i < n; ++i) {
        int32_t id = t.byte_id[s[i]];
        if (id < 0) continue;                       // byte without a token: dropped
        sy[m] = Sym{id, m - 1, m + 1, 1};
        ++m;
    }
    if (m == 0) return;
    sy[m - 1].next = -1;
    auto worse = [](const Cand& a, const Cand& b) { return a.rank > b.rank || (a.rank == b.rank && a.pos > b.pos); };
    q.clear();
    auto push = [&](int32_t pos) {
        int32_t nx = sy[pos].next;
        if (nx < 0) return;
        auto it = t.merges.find(((uint64_t)(uint32_t)sy[pos].id << 32) | (uint32_t)sy[nx].id);
        if (it == t.merges.end()) return;
        q.push_back({it->second.first, pos, it->second.second});
        std::push_heap(q.begin(), q.end(), worse);
    };
    for (int32_t i = 0; i + 1 < m; ++i) push(i);
    while (!q.empty()) {
        std::pop_heap(q.begin(), q.end(), worse);
        Cand c = q.back();
        q.pop_back();
        Sym& a = sy[c.pos];
        if (a.len == 0 || a.next < 0) continue;
        Sym& b = sy[a.next];
        auto it = t.merges.find(((uint64_t)(uint32_t)a.id << 32) | (uint32_t)b.id);
        if (it == t.merges.end() || it->second.second != c.id) continue;   // stale candidate
        a.id = c.id;
        a.len += b.len;
        b.len = 0;
        a.next = b.next;
        if (a.next >= 0) sy[a.next].prev = c.pos;
        if (a.prev >= 0) push(a.prev);
        push(c.pos);
    }
    for (int32_t i = 0; i >= 0; i = sy[i].next) out.push_back(sy[i].id);
}

// Normalised segment -> pieces -> ids.
void encode_normalized(const b2_tokenizer& t, const uint8_t* s, size_t n, std::vector<int32_t>& out,
                       std::vector<Ch>& chars) {
    chars.clear();
    for (size_t i = 0; i < n;) {
        size_t len;
        uint32_t cp = next_cp(s + i, n - i, &len);
        chars.push_back(Ch{cp, (uint32_t)i, char_class(cp)});
        i += len;
    }
    size_t nc = chars.size();
    for (size_t i = 0; i < nc;) {
        size_t k = match_piece(chars.data(), i, nc, t.pre);
        size_t b0 = chars[i].off, b1 = i + k < nc ? chars[i + k].off : n;
        bpe_piece(t, s + b0, b1 - b0, out);
        i += k;
    }
}

inline bool is_ws_cp(uint32_t cp) { return char_class(cp) == C_SPACE; }

// Splits s[0..n) on the added tokens of `trie` (longest match at the leftmost
// position); text between matches goes to `text(ptr, len)`, tokens to
// `tok(index)`.  A match that `ok` refuses (a special token the caller wants
// read as text) stays in the text and the scan resumes after it, as the HF
// library's encode_special_tokens does.  A single_word token's match stays
// text too when a word character touches it on either side.  lstrip /
// rstrip tokens take the whitespace beside them.
template <class Ok, class Text, class Tok>
void split_added(const b2_tokenizer& t, const Trie& trie, const uint8_t* s, size_t n, Ok ok, Text text, Tok tok) {
    if (trie.empty()) { text(s, n); return; }
    size_t seg = 0, i = 0;
    while (i < n) {
        size_t len = 0;
        int32_t idx = trie.longest(s + i, n - i, &len);
        if (idx < 0) { ++i; continue; }
        if (!ok(idx)) { i += len; continue; }
        size_t a = i, b = i + len;
        const AddedToken& at = t.added[idx];
        if (at.single_word) {
            bool word = false;
            if (a > 0) {
                size_t back = a - 1, l;
                while (back > 0 && a - back < 4 && (s[back] & 0xC0) == 0x80) --back;
                uint32_t cp = next_cp(s + back, n - back, &l);
                if (back + l != a) cp = kRawByte + s[a - 1];   // a stray continuation byte
                word = is_word_cp(cp);
            }
            if (!word && b < n) {
                size_t l;
                word = is_word_cp(next_cp(s + b, n - b, &l));
            }
            if (word) { i = b; continue; }
        }
        if (at.lstrip) {
            while (a > seg) {
                size_t back = a - 1;
                while (back > seg && (s[back] & 0xC0) == 0x80) --back;
                size_t l;
                if (!is_ws_cp(next_cp(s + back, n - back, &l))) break;
                a = back;
            }
        }
        if (at.rstrip) {
            while (b < n) {
                size_t l;
                if (!is_ws_cp(next_cp(s + b, n - b, &l))) break;
                b += l;
            }
        }
        if (a > seg) text(s + seg, a - seg);
        tok(idx);
        seg = i = b;
    }
    if (n > seg) text(s + seg, n - seg);
}

bool parse_template(b2_tokenizer& t, const JVal& pp) {
    const std::string* type = pp.str("type");
    if (!type) return true;
    if (*type == "Sequence") {
        const JVal* ps = pp.get("processors");
        if (ps && ps->t == JVal::ARR)
            for (auto& p : ps->arr)
                if (!parse_template(t, p)) return false;
        return true;
    }
    if (*type != "TemplateProcessing") return true;
    const JVal* single = pp.get("single");
    const JVal* specials = pp.get("special_tokens");
    if (!single || single->t != JVal::ARR) return false;
    bool seen_seq = false;
    for (auto& item : single->arr) {
        if (const JVal* sp = item.get("SpecialToken")) {
            const std::string* name = sp->str("id");
            if (!name || !specials) return false;
            const JVal* ent = specials->get(name->c_str());
            const JVal* ids = ent ? ent->get("ids") : nullptr;
            if (!ids || ids->t != JVal::ARR) return false;
            for (auto& v : ids->arr) (seen_seq ? t.suffix_ids : t.prefix_ids).push_back((int32_t)v.num);
        } else if (item.get("Sequence")) {
            seen_seq = true;
        }
    }
    t.has_template = true;
    return true;
}

int load_json(const char* text, size_t len, b2_tokenizer** out) {
    JVal root;
    JParser jp{text, text + len, {}};
    if (!jp.value(root, 0)) return tok_fail(B2_ERR_INVALID, "tokenizer.json: " + jp.err);
    std::unique_ptr<b2_tokenizer> t(new b2_tokenizer());

    // normalizer
    const JVal* norm = root.get("normalizer");
    if (norm && norm->t != JVal::NUL) {
        const std::string* ty = norm->str("type");
        if (ty && *ty == "NFC") t->use_nfc = true;
        else if (ty && *ty == "Sequence" && norm->get("normalizers") && norm->get("normalizers")->arr.empty()) {}
        else return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: normalizer other than NFC: " + (ty ? *ty : std::string("?")));
    }
    // pre_tokenizer
    const JVal* pre = root.get("pre_tokenizer");
    if (!pre || pre->t != JVal::OBJ) return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: no pre_tokenizer");
    std::vector<const JVal*> steps;
    if (const std::string* ty = pre->str("type"); ty && *ty == "Sequence") {
        const JVal* ps = pre->get("pretokenizers");
        if (!ps || ps->t != JVal::ARR) return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: bad pre_tokenizer sequence");
        for (auto& p : ps->arr) steps.push_back(&p);
    } else {
        steps.push_back(pre);
    }
    int kind = 0;
    bool byte_level = false;
    for (const JVal* st : steps) {
        const std::string* ty = st->str("type");
        if (!ty) return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: pre_tokenizer step without type");
        if (*ty == "Split") {
            const JVal* pat = st->get("pattern");
            const std::string* rx = pat ? pat->str("Regex") : nullptr;
            const std::string* beh = st->str("behavior");
            if (!rx || !beh || *beh != "Isolated" || st->is_true("invert") || kind)
                return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: Split step other than one isolated regex");
            if (*rx == kQwen2Pattern) kind = PRE_QWEN2;
            else if (*rx == kLlama3Pattern) kind = PRE_LLAMA3;
            else return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: unknown split pattern " + *rx);
        } else if (*ty == "ByteLevel") {
            if (st->is_true("add_prefix_space"))
                return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: ByteLevel add_prefix_space is not supported");
            const JVal* ur = st->get("use_regex");
            bool use_regex = !ur || ur->t != JVal::BOOL || ur->b;
            if (use_regex) {
                if (kind) return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: ByteLevel regex after a Split");
                kind = PRE_GPT2;
            }
            byte_level = true;
        } else {
            return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: pre_tokenizer " + *ty + " is not supported");
        }
    }
    if (!kind || !byte_level) return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: not a byte-level BPE pre-tokenizer");
    t->pre = kind;

    // model
    const JVal* model = root.get("model");
    if (!model || !model->str("type") || *model->str("type") != "BPE")
        return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: model is not BPE");
    if (model->is_true("byte_fallback")) return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: byte_fallback BPE");
    for (const char* k : {"continuing_subword_prefix", "end_of_word_suffix"}) {
        const std::string* v = model->str(k);
        if (v && !v->empty()) return tok_fail(B2_ERR_UNSUPPORTED, std::string("tokenizer.json: BPE ") + k);
    }
    if (const JVal* d = model->get("dropout"); d && d->t == JVal::NUM && d->num > 0)
        return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: BPE dropout");
    t->ignore_merges = model->is_true("ignore_merges");
    const JVal* vocab = model->get("vocab");
    if (!vocab || vocab->t != JVal::OBJ) return tok_fail(B2_ERR_INVALID, "tokenizer.json: model.vocab missing");
    int32_t max_id = -1;
    for (auto& kv : vocab->obj) max_id = std::max(max_id, (int32_t)kv.second.num);
    const JVal* addl = root.get("added_tokens");
    if (addl && addl->t == JVal::ARR)
        for (auto& a : addl->arr)
            if (const JVal* id = a.get("id")) max_id = std::max(max_id, (int32_t)id->num);
    t->id_bytes.assign((size_t)max_id + 1, std::string());
    t->id_special.assign((size_t)max_id + 1, 0);
    t->id_valid.assign((size_t)max_id + 1, 0);
    std::unordered_map<std::string, int32_t> by_string;   // as written in the file
    by_string.reserve(vocab->obj.size() * 2);
    t->vocab.reserve(vocab->obj.size() * 2);
    for (auto& kv : vocab->obj) {
        int32_t id = (int32_t)kv.second.num;
        if (kv.second.t != JVal::NUM || id < 0) return tok_fail(B2_ERR_INVALID, "tokenizer.json: bad vocab id");
        bool mapped;
        std::string bytes = token_bytes(kv.first, &mapped);
        if (mapped) t->vocab.emplace(bytes, id);
        t->id_bytes[id] = bytes;
        t->id_valid[id] = 1;
        by_string.emplace(kv.first, id);
    }
    for (int b = 0; b < 256; ++b) {
        auto it = t->vocab.find(std::string(1, (char)b));
        t->byte_id[b] = it == t->vocab.end() ? -1 : it->second;
    }
    const JVal* merges = model->get("merges");
    if (merges && merges->t == JVal::ARR) {
        t->merges.reserve(merges->arr.size() * 2);
        int32_t rank = 0;
        for (auto& m : merges->arr) {
            std::string a, b;
            if (m.t == JVal::STR) {
                size_t sp = m.s.find(' ', 1);
                if (sp == std::string::npos) return tok_fail(B2_ERR_INVALID, "tokenizer.json: merge without a space: " + m.s);
                a = m.s.substr(0, sp);
                b = m.s.substr(sp + 1);
            } else if (m.t == JVal::ARR && m.arr.size() == 2 && m.arr[0].t == JVal::STR && m.arr[1].t == JVal::STR) {
                a = m.arr[0].s;
                b = m.arr[1].s;
            } else {
                return tok_fail(B2_ERR_INVALID, "tokenizer.json: bad merge entry");
            }
            auto ia = by_string.find(a), ib = by_string.find(b), ic = by_string.find(a + b);
            if (ia == by_string.end() || ib == by_string.end() || ic == by_string.end())
                return tok_fail(B2_ERR_INVALID, "tokenizer.json: merge of tokens outside the vocab: " + a + " " + b);
            uint64_t key = ((uint64_t)(uint32_t)ia->second << 32) | (uint32_t)ib->second;
            t->merges.emplace(key, std::make_pair(rank, ic->second));   // first (lowest) rank wins
            ++rank;
        }
    }
    t->vocab_strings = by_string.size();

    // added tokens
    if (addl && addl->t == JVal::ARR) {
        for (auto& a : addl->arr) {
            AddedToken at;
            const std::string* content = a.str("content");
            const JVal* id = a.get("id");
            if (!content || !id || id->t != JVal::NUM || content->empty())
                return tok_fail(B2_ERR_INVALID, "tokenizer.json: bad added token");
            at.content = *content;
            at.id = (int32_t)id->num;
            at.special = a.is_true("special");
            at.normalized = a.is_true("normalized");
            at.lstrip = a.is_true("lstrip");
            at.rstrip = a.is_true("rstrip");
            at.single_word = a.is_true("single_word");
            bool mapped;
            t->id_bytes[at.id] = token_bytes(at.content, &mapped);
            t->id_special[at.id] = at.special;
            t->id_valid[at.id] = 1;
            if (!by_string.count(at.content)) ++t->vocab_strings;
            t->added_by_content[at.content] = at.id;
            int32_t idx = (int32_t)t->added.size();
            t->added.push_back(at);
            (at.normalized ? t->norm_trie : t->raw_trie).add(at.content, idx);
        }
    }

    // post-processor
    if (const JVal* pp = root.get("post_processor"); pp && pp->t == JVal::OBJ)
        if (!parse_template(*t, *pp)) return tok_fail(B2_ERR_UNSUPPORTED, "tokenizer.json: bad TemplateProcessing");

    // chat format and stop tokens
    auto find = [&](const char* s) -> int32_t {
        auto it = t->added_by_content.find(s);
        return it == t->added_by_content.end() ? -1 : it->second;
    };
    if (find("<|im_start|>") >= 0 && find("<|im_end|>") >= 0) {
        t->chat = B2_CHAT_CHATML;
        t->eos = find("<|im_end|>");
        t->stop.push_back(t->eos);
        if (find("<|endoftext|>") >= 0) t->stop.push_back(find("<|endoftext|>"));
    } else if (find("<|start_header_id|>") >= 0 && find("<|end_header_id|>") >= 0 && find("<|eot_id|>") >= 0) {
        t->chat = B2_CHAT_LLAMA3;
        t->eos = find("<|eot_id|>");
        t->bos = find("<|begin_of_text|>");
        t->stop.push_back(t->eos);
        if (find("<|end_of_text|>") >= 0) t->stop.push_back(find("<|end_of_text|>"));
        if (find("<|eom_id|>") >= 0) t->stop.push_back(find("<|eom_id|>"));
    } else if (find("<|endoftext|>") >= 0) {
        t->eos = find("<|endoftext|>");
        t->stop.push_back(t->eos);
    }
    if (t->bos < 0 && !t->prefix_ids.empty()) t->bos = t->prefix_ids[0];
    *out = t.release();
    return B2_OK;
}

// Python's str.strip() whitespace (what a Jinja `trim` removes).
inline bool py_space(uint32_t cp) {
    return (cp >= 0x09 && cp <= 0x0D) || (cp >= 0x1C && cp <= 0x20) || cp == 0x85 || cp == 0xA0 || cp == 0x1680 ||
           (cp >= 0x2000 && cp <= 0x200A) || cp == 0x2028 || cp == 0x2029 || cp == 0x202F || cp == 0x205F ||
           cp == 0x3000;
}

std::string py_strip(const std::string& s) {
    const uint8_t* p = (const uint8_t*)s.data();
    size_t n = s.size(), a = 0, b = n;
    while (a < n) {
        size_t l;
        uint32_t cp = next_cp(p + a, n - a, &l);
        if (!py_space(cp)) break;
        a += l;
    }
    size_t last_end = a;
    for (size_t i = a; i < n;) {
        size_t l;
        uint32_t cp = next_cp(p + i, n - i, &l);
        i += l;
        if (!py_space(cp)) last_end = i;
    }
    b = last_end;
    return s.substr(a, b - a);
}

int copy_out(const std::string& s, char* out, size_t cap, size_t* out_len) {
    *out_len = s.size();
    if (s.size() > cap) return tok_fail(B2_ERR_WORKSPACE, "output buffer too small");
    if (!s.empty()) memcpy(out, s.data(), s.size());
    return B2_OK;
}

}  // namespace

extern "C" {

int b2_tokenizer_load_json(const char* json, size_t len, b2_tokenizer** out) {
    if (!json || !out) return tok_fail(B2_ERR_INVALID, "null argument");
    *out = nullptr;
    return load_json(json, len, out);
}

int b2_tokenizer_load(const char* path, b2_tokenizer** out) {
    if (!path || !out) return tok_fail(B2_ERR_INVALID, "null argument");
    *out = nullptr;
    FILE* f = fopen(path, "rb");
    if (!f) return tok_fail(B2_ERR_INVALID, std::string("cannot open ") + path + ": " + strerror(errno));
    std::string buf;
    char chunk[1 << 16];
    size_t got;
    while ((got = fread(chunk, 1, sizeof(chunk), f)) > 0) buf.append(chunk, got);
    fclose(f);
    return load_json(buf.data(), buf.size(), out);
}

void b2_tokenizer_destroy(b2_tokenizer* t) { delete t; }

int b2_tokenizer_encode(const b2_tokenizer* t, const char* text, size_t len, int flags, int32_t* ids, size_t cap,
                        size_t* n_ids) {
    if (!t || (!text && len) || !n_ids || (!ids && cap)) return tok_fail(B2_ERR_INVALID, "null argument");
    std::vector<int32_t> out;
    out.reserve(len / 3 + 8);
    if (flags & B2_TOK_ADD_SPECIAL) out.insert(out.end(), t->prefix_ids.begin(), t->prefix_ids.end());
    const bool split_special = (flags & B2_TOK_SPLIT_SPECIAL) != 0;
    auto ok = [&](int32_t idx) { return split_special || !t->added[idx].special; };
    std::vector<Ch> chars;
    std::string normed;
    split_added(*t, t->raw_trie, (const uint8_t*)text, len, ok,
        [&](const uint8_t* s, size_t n) {
            if (t->use_nfc) {
                normed.clear();
                nfc(s, n, normed);
                s = (const uint8_t*)normed.data();
                n = normed.size();
            }
            split_added(*t, t->norm_trie, s, n, ok,
                [&](const uint8_t* p, size_t m) { encode_normalized(*t, p, m, out, chars); },
                [&](int32_t idx) { out.push_back(t->added[idx].id); });
        },
        [&](int32_t idx) { out.push_back(t->added[idx].id); });
    if (flags & B2_TOK_ADD_SPECIAL) out.insert(out.end(), t->suffix_ids.begin(), t->suffix_ids.end());
    *n_ids = out.size();
    if (out.size() > cap) return tok_fail(B2_ERR_WORKSPACE, "id buffer too small");
    if (!out.empty()) memcpy(ids, out.data(), out.size() * sizeof(int32_t));
    return B2_OK;
}

int b2_tokenizer_decode(const b2_tokenizer* t, const int32_t* ids, size_t n, int skip_special, char* out, size_t cap,
                        size_t* out_len) {
    if (!t || (!ids && n) || !out_len || (!out && cap)) return tok_fail(B2_ERR_INVALID, "null argument");
    std::string s;
    for (size_t i = 0; i < n; ++i) {
        int32_t id = ids[i];
        if (id < 0 || (size_t)id >= t->id_bytes.size() || !t->id_valid[id]) continue;
        if (skip_special && t->id_special[id]) continue;
        s += t->id_bytes[id];
    }
    return copy_out(s, out, cap, out_len);
}

int b2_tokenizer_apply_chat_template(const b2_tokenizer* t, const char* const* roles, const char* const* contents,
                                     size_t n_messages, int add_generation_prompt, char* out, size_t cap,
                                     size_t* out_len) {
    if (!t || !out_len || (!out && cap) || (n_messages && (!roles || !contents)))
        return tok_fail(B2_ERR_INVALID, "null argument");
    for (size_t i = 0; i < n_messages; ++i)
        if (!roles[i] || !contents[i]) return tok_fail(B2_ERR_INVALID, "null message field");
    std::string s;
    if (t->chat == B2_CHAT_CHATML) {
        size_t i = 0;
        if (n_messages && !strcmp(roles[0], "system")) {
            s += "<|im_start|>system\n";
            s += contents[0];
            s += "<|im_end|>\n";
            i = 1;
        } else {
            s += "<|im_start|>system\nYou are Qwen, created by Alibaba Cloud. You are a helpful assistant.<|im_end|>\n";
        }
        for (; i < n_messages; ++i) {
            s += "<|im_start|>";
            s += roles[i];
            s += "\n";
            s += contents[i];
            s += "<|im_end|>\n";
        }
        if (add_generation_prompt) s += "<|im_start|>assistant\n";
    } else if (t->chat == B2_CHAT_LLAMA3) {
        s += "<|begin_of_text|>";
        for (size_t i = 0; i < n_messages; ++i) {
            s += "<|start_header_id|>";
            s += roles[i];
            s += "<|end_header_id|>\n\n";
            s += py_strip(contents[i]);
            s += "<|eot_id|>";
        }
        if (add_generation_prompt) s += "<|start_header_id|>assistant<|end_header_id|>\n\n";
    } else {
        return tok_fail(B2_ERR_UNSUPPORTED, "no chat format for this vocabulary");
    }
    return copy_out(s, out, cap, out_len);
}

int b2_tokenizer_token_to_id(const b2_tokenizer* t, const char* token, size_t len, int32_t* id) {
    if (!t || !token || !id) return tok_fail(B2_ERR_INVALID, "null argument");
    std::string s(token, len);
    auto a = t->added_by_content.find(s);
    if (a != t->added_by_content.end()) { *id = a->second; return B2_OK; }
    bool mapped;
    std::string bytes = token_bytes(s, &mapped);
    auto v = mapped ? t->vocab.find(bytes) : t->vocab.end();
    if (v == t->vocab.end()) { *id = -1; return tok_fail(B2_ERR_INVALID, "no such token"); }
    *id = v->second;
    return B2_OK;
}

int b2_tokenizer_get_info(const b2_tokenizer* t, b2_tokenizer_info* info) {
    if (!t || !info) return tok_fail(B2_ERR_INVALID, "null argument");
    memset(info, 0, sizeof(*info));
    info->vocab_size = (int64_t)t->vocab_strings;
    info->n_ids = (int64_t)t->id_bytes.size();
    info->pre_tokenizer = t->pre;
    info->nfc = t->use_nfc;
    info->ignore_merges = t->ignore_merges;
    info->chat_format = t->chat;
    info->bos_id = t->bos;
    info->eos_id = t->eos;
    info->n_stop = (int32_t)std::min<size_t>(t->stop.size(), 4);
    for (int i = 0; i < 4; ++i) info->stop_ids[i] = i < info->n_stop ? t->stop[i] : -1;
    info->n_added = (int32_t)t->added.size();
    info->n_merges = (int64_t)t->merges.size();
    return B2_OK;
}

}  // extern "C"
