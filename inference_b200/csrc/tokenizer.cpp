// tokenizer.cpp -- the byte-level BPE tokenizer of Qwen3 checkpoints
// (tokenizer.json) and the text-level generate, host code behind the q3_*
// C ABI.
//
// Reference semantics followed (src/lib/tokenizer/tokenizer.cpp):
//   * tokenize (:217-235): the text is split at the added tokens (an
//     alternation of their strings, :40-87), which map to their ids; every
//     other piece is NFC-normalised (:103-118), split by the checkpoint's
//     pre-tokenizer pattern (:120-124), each byte of a split mapped to its
//     byte-level symbol (:126-134, alphabet :182-193), the symbols merged by
//     BPE -- repeatedly the leftmost occurrence of the adjacent pair of lowest
//     merge rank (:136-169) -- and looked up in the vocabulary (:89-101);
//   * decode (:237-265): added tokens verbatim, other tokens' symbols back to
//     their bytes;
//   * Generator::generate (src/lib/inference/generator.cpp:37-63): chat
//     template (src/lib/model/qwen3/qwen3.hpp:97-103), tokenize, prefill, greedy
//     decode until EOS or a full KV cache, decode the response.
// The reference matches the pattern with Boost.Regex over ICU and normalises
// with ICU.  Here the one pattern Qwen3 checkpoints carry (the Qwen2 split
// pattern; the loader checks the file holds exactly it) is matched by hand, and
// NFC and the \p{L} / \p{N} classes come from unicode_tables.inc (generated
// from the Unicode data by gen_unicode_tables.py).  BPE runs on token ids with
// a heap keyed by (merge rank, position): the reference's order of merges, in
// n log n instead of a rescan per merge.  The added tokens are tried longest
// first; the reference's alternation tries them in hash-map order, which
// agrees whenever no added token is a prefix of another (true of Qwen3's).
#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <queue>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "host_util.hpp"
#include "json.hpp"

namespace q3 {
namespace {

#include "unicode_tables.inc"

// ---------------------------------------------------------------- Unicode
template <class R>
bool in_ranges(const R* r, size_t n, uint32_t cp) {
    size_t lo = 0, hi = n;
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (cp < r[mid].lo) hi = mid;
        else if (cp > r[mid].hi) lo = mid + 1;
        else return true;
    }
    return false;
}
bool is_letter(uint32_t cp) { return in_ranges(kLetters, sizeof(kLetters) / sizeof(kLetters[0]), cp); }
bool is_number(uint32_t cp) { return in_ranges(kNumbers, sizeof(kNumbers) / sizeof(kNumbers[0]), cp); }
// What \s matches in the reference's pattern engine (Boost.Regex over ICU:
// u_isspace, general category Z plus TAB..CR, U+001C..U+001F and U+0085).
// Unlike the Unicode White_Space property it includes U+001C..U+001F.
bool is_space(uint32_t cp) {
    return (cp >= 0x09 && cp <= 0x0D) || (cp >= 0x1C && cp <= 0x20) || cp == 0x85 || cp == 0xA0 || cp == 0x1680 ||
           (cp >= 0x2000 && cp <= 0x200A) || cp == 0x2028 || cp == 0x2029 || cp == 0x202F || cp == 0x205F ||
           cp == 0x3000;
}
bool is_crlf(uint32_t cp) { return cp == '\r' || cp == '\n'; }

uint8_t ccc(uint32_t cp) {
    const size_t n = sizeof(kCcc) / sizeof(kCcc[0]);
    size_t lo = 0, hi = n;
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (cp < kCcc[mid].lo) hi = mid;
        else if (cp > kCcc[mid].hi) lo = mid + 1;
        else return kCcc[mid].ccc;
    }
    return 0;
}

// Hangul syllable arithmetic (the Unicode standard, section 3.12).
constexpr uint32_t kSBase = 0xAC00, kLBase = 0x1100, kVBase = 0x1161, kTBase = 0x11A7;
constexpr uint32_t kLCount = 19, kVCount = 21, kTCount = 28, kNCount = kVCount * kTCount, kSCount = kLCount * kNCount;

void decompose(uint32_t cp, std::vector<uint32_t>& out) {
    if (cp >= kSBase && cp < kSBase + kSCount) {
        const uint32_t s = cp - kSBase;
        out.push_back(kLBase + s / kNCount);
        out.push_back(kVBase + (s % kNCount) / kTCount);
        if (s % kTCount) out.push_back(kTBase + s % kTCount);
        return;
    }
    const size_t n = sizeof(kDecomp) / sizeof(kDecomp[0]);
    const Decomp* d = std::lower_bound(kDecomp, kDecomp + n, cp, [](const Decomp& x, uint32_t c) { return x.cp < c; });
    if (d != kDecomp + n && d->cp == cp) {
        decompose(d->a, out);
        if (d->b) decompose(d->b, out);
        return;
    }
    out.push_back(cp);
}

uint32_t compose_pair(uint32_t a, uint32_t b) {
    if (a >= kLBase && a < kLBase + kLCount && b >= kVBase && b < kVBase + kVCount)
        return kSBase + ((a - kLBase) * kVCount + (b - kVBase)) * kTCount;
    if (a >= kSBase && a < kSBase + kSCount && (a - kSBase) % kTCount == 0 && b > kTBase && b < kTBase + kTCount)
        return a + (b - kTBase);
    const size_t n = sizeof(kCompose) / sizeof(kCompose[0]);
    const Compose* c = std::lower_bound(kCompose, kCompose + n, std::make_pair(a, b),
                                        [](const Compose& x, const std::pair<uint32_t, uint32_t>& k) {
                                            return x.a < k.first || (x.a == k.first && x.b < k.second);
                                        });
    return (c != kCompose + n && c->a == a && c->b == b) ? c->cp : 0;
}

// NFC: canonical decomposition, canonical ordering, canonical composition.
std::vector<uint32_t> nfc(const std::vector<uint32_t>& in) {
    std::vector<uint32_t> d;
    d.reserve(in.size());
    for (uint32_t cp : in) decompose(cp, d);
    // stable sort of each run of non-starters by combining class
    for (size_t i = 0; i < d.size();) {
        if (ccc(d[i]) == 0) {
            ++i;
            continue;
        }
        size_t j = i;
        while (j < d.size() && ccc(d[j]) != 0) ++j;
        std::stable_sort(d.begin() + i, d.begin() + j, [](uint32_t x, uint32_t y) { return ccc(x) < ccc(y); });
        i = j;
    }
    std::vector<uint32_t> out;
    out.reserve(d.size());
    size_t starter = SIZE_MAX;  // index in out of the last starter
    int last_ccc = -1;          // combining class of the last code point after the starter
    for (uint32_t cp : d) {
        const int c = ccc(cp);
        if (starter != SIZE_MAX) {
            const bool blocked = last_ccc != -1 && (last_ccc == 0 || last_ccc >= c);
            if (!blocked) {
                const uint32_t comp = compose_pair(out[starter], cp);
                if (comp) {
                    out[starter] = comp;
                    continue;
                }
            }
        }
        if (c == 0) {
            starter = out.size();
            last_ccc = -1;
        } else {
            last_ccc = c;
        }
        out.push_back(cp);
    }
    return out;
}

// ---------------------------------------------------------------- UTF-8
// UTF-8 to code points.  Ill-formed input becomes U+FFFD, one per maximal
// subpart of an ill-formed sequence (the Unicode standard's recommended
// practice, section 3.9, which ICU's UTF-8 conversion in the reference and
// Python's "replace" error handler both follow).
void utf8_decode(const std::string& s, std::vector<uint32_t>& out) {
    const size_t n = s.size();
    for (size_t i = 0; i < n;) {
        const unsigned c = static_cast<unsigned char>(s[i]);
        if (c < 0x80) {
            out.push_back(c);
            ++i;
            continue;
        }
        int len = 0;
        unsigned lo = 0x80, hi = 0xBF;  // the allowed range of the second byte
        uint32_t cp = 0;
        if (c >= 0xC2 && c <= 0xDF) {
            len = 2;
            cp = c & 0x1F;
        } else if (c >= 0xE0 && c <= 0xEF) {
            len = 3;
            cp = c & 0x0F;
            if (c == 0xE0) lo = 0xA0;
            if (c == 0xED) hi = 0x9F;
        } else if (c >= 0xF0 && c <= 0xF4) {
            len = 4;
            cp = c & 0x07;
            if (c == 0xF0) lo = 0x90;
            if (c == 0xF4) hi = 0x8F;
        }
        if (len == 0) {  // a continuation byte without a lead, C0, C1, F5..FF
            out.push_back(0xFFFD);
            ++i;
            continue;
        }
        size_t k = 1;
        for (; k < static_cast<size_t>(len) && i + k < n; ++k) {
            const unsigned t = static_cast<unsigned char>(s[i + k]);
            if (k == 1 ? (t < lo || t > hi) : (t < 0x80 || t > 0xBF)) break;
            cp = (cp << 6) | (t & 0x3F);
        }
        out.push_back(k == static_cast<size_t>(len) ? cp : 0xFFFD);
        i += k;
    }
}

// ---------------------------------------------------------------- pre-tokenizer
// The Qwen2 split pattern, the one Qwen3's tokenizer.json carries:
//   (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+
// matched by hand at each position: the first alternative that matches wins,
// each with its greedy quantifiers backtracked as a regex engine would.
const char kQwen2Pattern[] =
    "(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}| ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*|"
    "\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+";

size_t match_at(const std::vector<uint32_t>& c, size_t i) {
    const size_t n = c.size();
    // simple case folding onto the ASCII letters of the contractions: A-Z and
    // U+017F (long s, which folds to 's'); U+212A (Kelvin) folds to 'k', unused
    auto lower = [](uint32_t x) -> uint32_t { return (x >= 'A' && x <= 'Z') ? x + 32 : x == 0x17F ? 's' : x; };
    // 1. contractions, case-insensitive
    if (c[i] == '\'' && i + 1 < n) {
        const uint32_t a = lower(c[i + 1]), b = i + 2 < n ? lower(c[i + 2]) : 0;
        if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
        if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
    }
    // 2. [^\r\n\p{L}\p{N}]?\p{L}+
    {
        size_t j = i;
        if (!is_crlf(c[j]) && !is_letter(c[j]) && !is_number(c[j]) && j + 1 < n && is_letter(c[j + 1])) ++j;
        if (is_letter(c[j])) {
            while (j < n && is_letter(c[j])) ++j;
            return j - i;
        }
    }
    // 3. \p{N}
    if (is_number(c[i])) return 1;
    // 4.  ?[^\s\p{L}\p{N}]+[\r\n]*
    {
        auto other = [&](uint32_t x) { return !is_space(x) && !is_letter(x) && !is_number(x); };
        size_t j = i;
        if (c[j] == ' ' && j + 1 < n && other(c[j + 1])) ++j;
        if (other(c[j])) {
            while (j < n && other(c[j])) ++j;
            while (j < n && is_crlf(c[j])) ++j;
            return j - i;
        }
    }
    // the whitespace run at i
    size_t run = i;
    while (run < n && is_space(c[run])) ++run;
    if (run > i) {
        // 5. \s*[\r\n]+ : up to the last CR / LF of the run
        for (size_t k = run; k > i; --k)
            if (is_crlf(c[k - 1])) return k - i;
        // 6. \s+(?!\S) : the run, or all of it but its last character when text follows
        if (run == n) return run - i;
        if (run - i >= 2) return run - 1 - i;
        // 7. \s+
        return run - i;
    }
    return 1;  // not reached: every code point is a letter, a number, a space or "other"
}

// ---------------------------------------------------------------- the tokenizer
struct PairHash {
    size_t operator()(uint64_t k) const noexcept { return std::hash<uint64_t>()(k * 0x9E3779B97F4A7C15ull); }
};

}  // namespace
}  // namespace q3

struct q3_tokenizer {
    std::unordered_map<std::string, uint32_t> vocab;
    std::vector<std::string> id_to_word;                  // by id; empty where unused
    std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>, q3::PairHash> merges;  // (left, right) -> (rank, merged)
    std::vector<std::pair<std::string, uint32_t>> special;  // added tokens, longest first
    std::unordered_map<uint32_t, std::string> special_by_id;
    uint32_t byte_id[256] = {};                            // the byte-level symbol of each byte, as an id
    std::unordered_map<uint32_t, uint8_t> cp_to_byte;      // byte-level code point -> byte
};

namespace q3 {
namespace {

// The byte-level alphabet (tokenizer.cpp:183-194): printable Latin-1 bytes
// keep their code point, the others map to U+0100 upwards in byte order.
uint32_t byte_codepoint(unsigned b, uint32_t& next) {
    const bool keep = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
    return keep ? b : next++;
}

int load(const std::string& path_in, q3_tokenizer& t) {
    std::string path = path_in;
    {
        std::ifstream probe(path + "/tokenizer.json", std::ios::binary);
        if (probe) path += "/tokenizer.json";
    }
    std::ifstream f(path, std::ios::binary);
    if (!f) return fail(Q3_ERR_INVALID, "cannot open " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    const std::string text = ss.str();
    Json j;
    std::string err;
    if (!parse_json(text.data(), text.size(), j, err) || j.kind != Json::Obj)
        return fail(Q3_ERR_INVALID, path + ": JSON: " + (err.empty() ? "not an object" : err));
    const Json* model = j.get("model");
    const Json* vocab = model ? model->get("vocab") : nullptr;
    const Json* merges = model ? model->get("merges") : nullptr;
    const Json* type = model ? model->get("type") : nullptr;
    if (!vocab || vocab->kind != Json::Obj || !merges || merges->kind != Json::Arr)
        return fail(Q3_ERR_INVALID, path + ": no model.vocab / model.merges");
    if (type && type->kind == Json::Str && type->str != "BPE")
        return fail(Q3_ERR_UNSUPPORTED, path + ": model type " + type->str + " (BPE only)");
    // the pre-tokenizer must be the pattern this file implements
    const Json* pre = j.get("pre_tokenizer");
    const Json* seq = pre ? pre->get("pretokenizers") : nullptr;
    const Json* first = (seq && seq->kind == Json::Arr && !seq->arr.empty()) ? &seq->arr[0] : nullptr;
    const Json* pat = first ? first->get("pattern") : nullptr;
    const Json* rx = pat ? pat->get("Regex") : nullptr;
    if (!rx || rx->kind != Json::Str || rx->str != kQwen2Pattern)
        return fail(Q3_ERR_UNSUPPORTED, path + ": pre-tokenizer pattern is not the Qwen2 split pattern");
    // ids are integers below 2^24 (Qwen3's vocabularies hold ~152k)
    auto valid_id = [](const Json* v) {
        return v && v->kind == Json::Num && v->num >= 0 && v->num < 16777216.0 &&
               v->num == static_cast<double>(static_cast<uint32_t>(v->num));
    };
    uint32_t max_id = 0;
    t.vocab.reserve(vocab->obj.size());
    for (const auto& kv : vocab->obj) {
        if (!valid_id(&kv.second)) return fail(Q3_ERR_INVALID, path + ": bad vocabulary id for " + kv.first);
        const uint32_t id = static_cast<uint32_t>(kv.second.num);
        t.vocab.emplace(kv.first, id);
        max_id = std::max(max_id, id);
    }
    const Json* added = j.get("added_tokens");
    if (added && added->kind == Json::Arr) {
        for (const Json& a : added->arr) {
            const Json* id = a.get("id");
            const Json* content = a.get("content");
            if (!valid_id(id) || !content || content->kind != Json::Str || content->str.empty())
                return fail(Q3_ERR_INVALID, path + ": malformed added token");
            const uint32_t v = static_cast<uint32_t>(id->num);
            t.special.emplace_back(content->str, v);
            t.special_by_id[v] = content->str;
            max_id = std::max(max_id, v);
        }
    }
    std::stable_sort(t.special.begin(), t.special.end(),
                     [](const auto& a, const auto& b) { return a.first.size() > b.first.size(); });
    t.id_to_word.assign(static_cast<size_t>(max_id) + 1, std::string());
    for (const auto& kv : t.vocab) t.id_to_word[kv.second] = kv.first;
    // byte-level symbols as ids
    uint32_t next = 0x100;
    for (unsigned b = 0; b < 256; ++b) {
        const uint32_t cp = byte_codepoint(b, next);
        std::string sym;
        append_utf8(sym, cp);
        const auto it = t.vocab.find(sym);
        if (it == t.vocab.end()) return fail(Q3_ERR_INVALID, path + ": vocabulary lacks a byte-level symbol");
        t.byte_id[b] = it->second;
        t.cp_to_byte[cp] = static_cast<uint8_t>(b);
    }
    // merges: "left right" strings (older files) or [left, right] pairs
    t.merges.reserve(merges->arr.size());
    for (size_t r = 0; r < merges->arr.size(); ++r) {
        const Json& m = merges->arr[r];
        std::string left, right;
        if (m.kind == Json::Arr && m.arr.size() == 2 && m.arr[0].kind == Json::Str && m.arr[1].kind == Json::Str) {
            left = m.arr[0].str;
            right = m.arr[1].str;
        } else if (m.kind == Json::Str && m.str.find(' ') != std::string::npos) {
            left = m.str.substr(0, m.str.find(' '));
            right = m.str.substr(m.str.find(' ') + 1);
        } else {
            return fail(Q3_ERR_INVALID, path + ": malformed merge " + std::to_string(r));
        }
        const auto l = t.vocab.find(left), rr = t.vocab.find(right), lr = t.vocab.find(left + right);
        if (l == t.vocab.end() || rr == t.vocab.end() || lr == t.vocab.end()) continue;  // can never apply
        const uint64_t key = (static_cast<uint64_t>(l->second) << 32) | rr->second;
        t.merges.emplace(key, std::make_pair(static_cast<uint32_t>(r), lr->second));  // the first rank wins
    }
    return Q3_OK;
}

// BPE over the byte-level ids of one pre-tokenizer split.
void bpe(const q3_tokenizer& t, std::vector<uint32_t>& sym) {
    const size_t n = sym.size();
    if (n < 2) return;
    std::vector<int> prev(n), next(n);
    std::vector<char> alive(n, 1);
    for (size_t i = 0; i < n; ++i) {
        prev[i] = static_cast<int>(i) - 1;
        next[i] = i + 1 < n ? static_cast<int>(i + 1) : -1;
    }
    using Item = std::pair<uint64_t, uint32_t>;  // (rank << 32 | left position, right symbol when queued)
    std::priority_queue<Item, std::vector<Item>, std::greater<Item>> heap;
    auto push = [&](int i) {
        if (i < 0 || next[i] < 0) return;
        const auto it = t.merges.find((static_cast<uint64_t>(sym[i]) << 32) | sym[next[i]]);
        if (it != t.merges.end())
            heap.emplace((static_cast<uint64_t>(it->second.first) << 32) | static_cast<uint32_t>(i), sym[next[i]]);
    };
    for (size_t i = 0; i + 1 < n; ++i) push(static_cast<int>(i));
    while (!heap.empty()) {
        const Item top = heap.top();
        heap.pop();
        const int i = static_cast<int>(top.first & 0xFFFFFFFFu);
        const uint32_t rank = static_cast<uint32_t>(top.first >> 32);
        if (!alive[i] || next[i] < 0 || sym[next[i]] != top.second) continue;  // stale entry
        const auto it = t.merges.find((static_cast<uint64_t>(sym[i]) << 32) | sym[next[i]]);
        if (it == t.merges.end() || it->second.first != rank) continue;
        const int j = next[i];
        sym[i] = it->second.second;
        alive[j] = 0;
        next[i] = next[j];
        if (next[j] >= 0) prev[next[j]] = i;
        push(prev[i]);
        push(i);
    }
    std::vector<uint32_t> out;
    for (int i = 0; i >= 0; i = next[i]) out.push_back(sym[i]);
    sym.swap(out);
}

int encode_text(const q3_tokenizer& t, const std::string& text, std::vector<uint32_t>& ids) {
    std::vector<uint32_t> cps;
    utf8_decode(text, cps);
    cps = nfc(cps);
    for (size_t i = 0; i < cps.size();) {
        const size_t len = match_at(cps, i);
        std::string piece;
        for (size_t k = i; k < i + len; ++k) append_utf8(piece, cps[k]);
        std::vector<uint32_t> sym;
        sym.reserve(piece.size());
        for (unsigned char b : piece) sym.push_back(t.byte_id[b]);
        bpe(t, sym);
        ids.insert(ids.end(), sym.begin(), sym.end());
        i += len;
    }
    return Q3_OK;
}

int encode(const q3_tokenizer& t, const std::string& text, std::vector<uint32_t>& ids) {
    size_t start = 0;
    for (size_t i = 0; i < text.size();) {
        const std::pair<std::string, uint32_t>* hit = nullptr;
        for (const auto& s : t.special)  // longest first
            if (text.compare(i, s.first.size(), s.first) == 0) {
                hit = &s;
                break;
            }
        if (!hit) {
            ++i;
            continue;
        }
        if (i > start) Q3_TRY_STATUS(encode_text(t, text.substr(start, i - start), ids));
        ids.push_back(hit->second);
        i += hit->first.size();
        start = i;
    }
    if (start < text.size()) Q3_TRY_STATUS(encode_text(t, text.substr(start), ids));
    return Q3_OK;
}

int decode(const q3_tokenizer& t, const uint32_t* ids, size_t n, std::string& out) {
    for (size_t k = 0; k < n; ++k) {
        const auto sp = t.special_by_id.find(ids[k]);
        if (sp != t.special_by_id.end()) {
            out += sp->second;
            continue;
        }
        if (ids[k] >= t.id_to_word.size() || t.id_to_word[ids[k]].empty())
            return fail(Q3_ERR_INVALID, "token id " + std::to_string(ids[k]) + " is not in the vocabulary");
        std::vector<uint32_t> cps;
        utf8_decode(t.id_to_word[ids[k]], cps);
        for (uint32_t cp : cps) {
            const auto b = t.cp_to_byte.find(cp);
            if (b == t.cp_to_byte.end())
                return fail(Q3_ERR_INVALID, "token contains a character outside the byte-level alphabet");
            out += static_cast<char>(b->second);
        }
    }
    return Q3_OK;
}

// The Qwen3 chat template of the reference (qwen3.hpp:97-103).
std::string chat_template(const std::string& prompt) {
    return "<|im_start|>user\n" + prompt + "<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>";
}

int copy_out(const std::string& s, char* out, size_t capacity, size_t* needed) {
    if (needed) *needed = s.size() + 1;
    if (!out) return Q3_OK;
    if (capacity < s.size() + 1) return fail(Q3_ERR_INVALID, "output buffer too small");
    std::memcpy(out, s.data(), s.size());
    out[s.size()] = '\0';
    return Q3_OK;
}

// q3_engine_generate_text after its argument checks.
int generate_text(q3_engine* e, const q3_tokenizer* t, const char* prompt, size_t len, char** out,
                  size_t* out_len) {
    std::vector<uint32_t> ids;
    Q3_TRY_STATUS(encode(*t, chat_template(std::string(prompt ? prompt : "", len)), ids));
    // generator.cpp:42-44 (q3_engine_generate checks it too)
    if (ids.size() >= engine_capacity(e)) return fail(Q3_ERR_INVALID, "prompt does not fit in the model context");
    // greedy decode until EOS (not emitted) or a full cache (generator.cpp:49-56)
    std::vector<uint32_t> gen(engine_capacity(e));
    size_t n = 0;
    Q3_TRY_STATUS(q3_engine_generate(e, ids.data(), ids.size(), gen.size(), /*stop_at_eos=*/1, gen.data(), &n));
    std::string s;
    Q3_TRY_STATUS(decode(*t, gen.data(), n, s));
    char* buf = static_cast<char*>(std::malloc(s.size() + 1));
    if (!buf) return fail(Q3_ERR_OOM, "q3_engine_generate_text: host allocation failed");
    std::memcpy(buf, s.data(), s.size());
    buf[s.size()] = '\0';
    *out = buf;
    *out_len = s.size();
    return Q3_OK;
}

}  // namespace
}  // namespace q3

using namespace q3;

extern "C" {

int q3_tokenizer_load(const char* path, q3_tokenizer** out) {
    Q3_CHECK(path && out, "q3_tokenizer_load: null argument");
    *out = nullptr;
    return guarded("q3_tokenizer_load", [&]() -> int {
        auto t = std::make_unique<q3_tokenizer>();
        const int rc = load(path, *t);
        if (rc == Q3_OK) *out = t.release();
        return rc;
    });
}

int q3_tokenizer_destroy(q3_tokenizer* t) {
    delete t;
    return Q3_OK;
}

int q3_tokenizer_encode(const q3_tokenizer* t, const char* text, size_t len, uint32_t* ids, size_t capacity,
                        size_t* n_ids) {
    Q3_CHECK(t && (text || len == 0) && n_ids, "q3_tokenizer_encode: null argument");
    return guarded("q3_tokenizer_encode", [&]() -> int {
        std::vector<uint32_t> v;
        const int rc = encode(*t, std::string(text ? text : "", len), v);
        if (rc != Q3_OK) return rc;
        *n_ids = v.size();
        if (!ids) return Q3_OK;
        Q3_CHECK(capacity >= v.size(), "q3_tokenizer_encode: ids buffer too small");
        std::copy(v.begin(), v.end(), ids);
        return Q3_OK;
    });
}

int q3_tokenizer_decode(const q3_tokenizer* t, const uint32_t* ids, size_t n, char* out, size_t capacity,
                        size_t* needed) {
    Q3_CHECK(t && (ids || n == 0), "q3_tokenizer_decode: null argument");
    return guarded("q3_tokenizer_decode", [&]() -> int {
        std::string s;
        const int rc = decode(*t, ids, n, s);
        if (rc != Q3_OK) return rc;
        return copy_out(s, out, capacity, needed);
    });
}

int q3_chat_template(const char* prompt, size_t len, char* out, size_t capacity, size_t* needed) {
    Q3_CHECK(prompt || len == 0, "q3_chat_template: null argument");
    return guarded("q3_chat_template",
                   [&]() -> int {
                       return copy_out(chat_template(std::string(prompt ? prompt : "", len)), out, capacity, needed);
                   });
}

int q3_engine_generate_text(q3_engine* e, const q3_tokenizer* t, const char* prompt, size_t len, char** out,
                            size_t* out_len) {
    Q3_CHECK(e && t && (prompt || len == 0) && out && out_len, "q3_engine_generate_text: null argument");
    *out = nullptr;
    *out_len = 0;
    return guarded("q3_engine_generate_text",
                   [&]() -> int { return generate_text(e, t, prompt, len, out, out_len); });
}

void q3_string_free(char* s) { std::free(s); }

}  // extern "C"
