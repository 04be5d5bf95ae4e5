// Llama-3 byte-level BPE tokenizer (host code behind the C ABI).
//
// Replaces the reference's Tokenizer (inferencer.cu:361-451) with the same
// results: the same Unicode pre-tokenizer pattern (PCRE2 with UTF and UCP, as
// the reference compiles it), each piece's bytes mapped to the GGUF byte
// symbols (bytes 33-126, 161-172 and 174-255 stand for themselves, the others
// for code points 256, 257, ... in byte order), then merges applied lowest
// rank first, leftmost first among equal ranks, until none applies.
//
// What differs is the cost.  The reference matches every piece with PCRE2
// (which re-checks the rest of the text's UTF-8 on each call) and rebuilds a
// "left right" string and hashes it for every adjacent pair on every merge
// step.  Here valid UTF-8 is checked once and split by a scanner that walks
// the pattern's alternatives over character classes probed from PCRE2 itself
// (scan_piece); merges are a flat hash table from a pair of token ids to
// (rank, merged id), a piece of up to kScanMax symbols merged in an array that keeps
// each adjacent pair's rank, a longer one through a min-heap of (rank,
// position) entries over a linked list; and pieces already seen are served
// from a flat per-thread cache.  PCRE2 (loaded from libpcre2-8.so.0 when the
// first tokenizer is created) still matches text that is not valid UTF-8,
// exactly as the reference matches it.
#include <dlfcn.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <memory>
#include <mutex>
#include <queue>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/ijb200.h"

namespace {

// ------------------------------------------------------------------ PCRE2 --
// The 8-bit entry points and option values of PCRE2's public API.
struct Pcre2 {
    void *(*compile)(const uint8_t *, size_t, uint32_t, int *, size_t *, void *) = nullptr;
    int (*jit_compile)(void *, uint32_t) = nullptr;
    void *(*match_data_create)(const void *, void *) = nullptr;
    int (*match)(const void *, const uint8_t *, size_t, size_t, uint32_t, void *, void *) = nullptr;
    size_t *(*ovector)(void *) = nullptr;
    void (*match_data_free)(void *) = nullptr;
    void (*code_free)(void *) = nullptr;
};
constexpr uint32_t kPcre2Ucp = 0x00020000u, kPcre2Utf = 0x00080000u, kPcre2NoUtfCheck = 0x40000000u;
constexpr uint32_t kPcre2JitComplete = 0x00000001u;
constexpr size_t kPcre2ZeroTerminated = ~static_cast<size_t>(0);

const Pcre2 &pcre2() {
    static Pcre2 api;
    static std::once_flag once;
    static std::string error;
    std::call_once(once, [] {
        void *lib = dlopen("libpcre2-8.so.0", RTLD_NOW | RTLD_LOCAL);
        if (!lib) {
            error = "PCRE2 runtime library (libpcre2-8.so.0) not found";
            return;
        }
        auto sym = [&](const char *name) { return dlsym(lib, name); };
        api.compile = reinterpret_cast<decltype(api.compile)>(sym("pcre2_compile_8"));
        api.jit_compile = reinterpret_cast<decltype(api.jit_compile)>(sym("pcre2_jit_compile_8"));
        api.match_data_create =
            reinterpret_cast<decltype(api.match_data_create)>(sym("pcre2_match_data_create_from_pattern_8"));
        api.match = reinterpret_cast<decltype(api.match)>(sym("pcre2_match_8"));
        api.ovector = reinterpret_cast<decltype(api.ovector)>(sym("pcre2_get_ovector_pointer_8"));
        api.match_data_free = reinterpret_cast<decltype(api.match_data_free)>(sym("pcre2_match_data_free_8"));
        api.code_free = reinterpret_cast<decltype(api.code_free)>(sym("pcre2_code_free_8"));
        if (!api.compile || !api.match_data_create || !api.match || !api.ovector || !api.match_data_free ||
            !api.code_free)
            error = "PCRE2 runtime library lacks its 8-bit API";
    });
    if (!error.empty()) throw std::runtime_error(error);
    return api;
}

// Llama 3's pre-tokenizer (the pattern inferencer.cu:379-383 compiles).
const char *const kPattern =
    "(?:'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD])|"
    "[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}{1,3}|"
    " ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*|\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+";

// Strict UTF-8 (RFC 3629: no overlong forms, no surrogates, nothing above
// U+10FFFF) — the check PCRE2 applies to a UTF subject.
bool valid_utf8(const uint8_t *s, size_t n) {
    size_t i = 0;
    while (i < n) {
        const uint8_t c = s[i];
        if (c < 0x80) {
            ++i;
            continue;
        }
        int len;
        uint32_t cp;
        if (c >= 0xc2 && c <= 0xdf) {
            len = 2;
            cp = c & 0x1f;
        } else if (c >= 0xe0 && c <= 0xef) {
            len = 3;
            cp = c & 0x0f;
        } else if (c >= 0xf0 && c <= 0xf4) {
            len = 4;
            cp = c & 0x07;
        } else {
            return false;
        }
        if (i + len > n) return false;
        for (int k = 1; k < len; ++k) {
            const uint8_t t = s[i + k];
            if ((t & 0xc0) != 0x80) return false;
            cp = (cp << 6) | (t & 0x3f);
        }
        if ((len == 3 && cp < 0x800) || (len == 4 && (cp < 0x10000 || cp > 0x10ffff)) ||
            (cp >= 0xd800 && cp <= 0xdfff))
            return false;
        i += len;
    }
    return true;
}

std::string utf8_of(uint32_t cp) {
    std::string s;
    if (cp < 0x80) {
        s.push_back(static_cast<char>(cp));
    } else if (cp < 0x800) {
        s.push_back(static_cast<char>(0xc0 | (cp >> 6)));
        s.push_back(static_cast<char>(0x80 | (cp & 63)));
    } else {
        s.push_back(static_cast<char>(0xe0 | (cp >> 12)));
        s.push_back(static_cast<char>(0x80 | ((cp >> 6) & 63)));
        s.push_back(static_cast<char>(0x80 | (cp & 63)));
    }
    return s;
}

// Character classes of the pattern (PCRE2 with UTF + UCP) for every code
// point, probed once per process from PCRE2 itself: the runs that \p{L}+,
// \p{N}+ and \s+ match over a string of all code points in order.  So the
// scanner below classifies each character exactly as the matcher would, in
// whatever Unicode version the installed PCRE2 carries.
enum : uint8_t { kOtherCls = 0, kLetterCls = 1, kDigitCls = 2, kSpaceCls = 3, kNewlineCls = 4 };
constexpr uint32_t kMaxCp = 0x110000;

const std::vector<uint8_t> *code_point_classes() {
    static std::vector<uint8_t> cls;
    static std::once_flag once;
    static bool ok = false;
    std::call_once(once, [] {
        const Pcre2 &api = pcre2();
        std::string all;
        std::vector<uint32_t> start;  // byte offset of each code point in `all` (surrogates skipped)
        std::vector<uint32_t> cps;
        all.reserve(4u << 20);
        for (uint32_t cp = 0; cp < kMaxCp; ++cp) {
            if (cp >= 0xd800 && cp <= 0xdfff) continue;
            start.push_back(static_cast<uint32_t>(all.size()));
            cps.push_back(cp);
            if (cp < 0x80) {
                all.push_back(static_cast<char>(cp));
            } else if (cp < 0x800) {
                all.push_back(static_cast<char>(0xc0 | (cp >> 6)));
                all.push_back(static_cast<char>(0x80 | (cp & 63)));
            } else if (cp < 0x10000) {
                all.push_back(static_cast<char>(0xe0 | (cp >> 12)));
                all.push_back(static_cast<char>(0x80 | ((cp >> 6) & 63)));
                all.push_back(static_cast<char>(0x80 | (cp & 63)));
            } else {
                all.push_back(static_cast<char>(0xf0 | (cp >> 18)));
                all.push_back(static_cast<char>(0x80 | ((cp >> 12) & 63)));
                all.push_back(static_cast<char>(0x80 | ((cp >> 6) & 63)));
                all.push_back(static_cast<char>(0x80 | (cp & 63)));
            }
        }
        cls.assign(kMaxCp, kOtherCls);
        const uint8_t *subject = reinterpret_cast<const uint8_t *>(all.data());
        auto index_of = [&](size_t off) {
            return static_cast<size_t>(std::lower_bound(start.begin(), start.end(), static_cast<uint32_t>(off)) -
                                       start.begin());
        };
        const std::pair<const char *, uint8_t> probes[] = {
            {"\\p{L}+", kLetterCls}, {"\\p{N}+", kDigitCls}, {"\\s+", kSpaceCls}};
        for (const auto &[pattern, value] : probes) {
            int err = 0;
            size_t off = 0;
            void *code = api.compile(reinterpret_cast<const uint8_t *>(pattern), kPcre2ZeroTerminated,
                                     kPcre2Utf | kPcre2Ucp, &err, &off, nullptr);
            if (!code) return;
            if (api.jit_compile) api.jit_compile(code, kPcre2JitComplete);
            void *md = api.match_data_create(code, nullptr);
            if (!md) {
                api.code_free(code);
                return;
            }
            for (size_t pos = 0; pos < all.size();) {
                if (api.match(code, subject, all.size(), pos, kPcre2NoUtfCheck, md, nullptr) < 0) break;
                const size_t *span = api.ovector(md);
                for (size_t k = index_of(span[0]); k < cps.size() && start[k] < span[1]; ++k) cls[cps[k]] = value;
                pos = span[1] > span[0] ? span[1] : span[1] + 1;
            }
            api.match_data_free(md);
            api.code_free(code);
        }
        cls['\r'] = kNewlineCls;
        cls['\n'] = kNewlineCls;
        // the classes the pattern's ASCII reading takes for granted
        ok = cls['a'] == kLetterCls && cls['Z'] == kLetterCls && cls['7'] == kDigitCls && cls[' '] == kSpaceCls &&
             cls['\t'] == kSpaceCls && cls['\''] == kOtherCls;
    });
    return ok ? &cls : nullptr;
}

// One code point of valid UTF-8 at t[k] (k < n): its value, *len its bytes.
inline uint32_t decode_cp(const uint8_t *t, size_t k, uint32_t *len) {
    const uint8_t c = t[k];
    if (c < 0x80) {
        *len = 1;
        return c;
    }
    if (c < 0xe0) {
        *len = 2;
        return (static_cast<uint32_t>(c & 0x1f) << 6) | (t[k + 1] & 0x3f);
    }
    if (c < 0xf0) {
        *len = 3;
        return (static_cast<uint32_t>(c & 0x0f) << 12) | (static_cast<uint32_t>(t[k + 1] & 0x3f) << 6) |
               (t[k + 2] & 0x3f);
    }
    *len = 4;
    return (static_cast<uint32_t>(c & 0x07) << 18) | (static_cast<uint32_t>(t[k + 1] & 0x3f) << 12) |
           (static_cast<uint32_t>(t[k + 2] & 0x3f) << 6) | (t[k + 3] & 0x3f);
}

// The pattern's match at position i of valid UTF-8 text, found without PCRE2:
// its seven alternatives in their order, each with the backtracking PCRE2
// would do (the optional leading character of the letter and punctuation
// alternatives given back when what follows does not match, \s*[\r\n]+ ending
// at a whitespace run's last CR or LF, \s+(?!\S) giving back a run's last
// character when a non-space follows).  Every position of valid UTF-8 starts a
// match, so the pieces are the matches, back to back.
size_t scan_piece(const uint8_t *t, size_t n, size_t i, const uint8_t *cls) {
    uint32_t len0;
    const uint32_t c0 = decode_cp(t, i, &len0);
    const uint8_t k0 = cls[c0];
    auto cls_at = [&](size_t k, uint32_t *len) { return cls[decode_cp(t, k, len)]; };
    auto run = [&](size_t k, uint8_t want) {  // end of a run of class `want` from k
        uint32_t len;
        while (k < n && cls_at(k, &len) == want) k += len;
        return k;
    };
    // '[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD]
    if (c0 == '\'' && i + 1 < n) {
        const uint8_t a = t[i + 1] | 0x20;  // lower case of an ASCII letter; no other byte maps onto these
        if (a == 's' || a == 't' || a == 'm' || a == 'd') return i + 2;
        if (i + 2 < n) {
            const uint8_t b = t[i + 2] | 0x20;
            if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return i + 3;
        }
    }
    // [^\r\n\p{L}\p{N}]?\p{L}+
    if (k0 == kLetterCls) return run(i, kLetterCls);
    if (k0 == kOtherCls || k0 == kSpaceCls) {
        uint32_t len;
        if (i + len0 < n && cls_at(i + len0, &len) == kLetterCls) return run(i + len0, kLetterCls);
    }
    // \p{N}{1,3}
    if (k0 == kDigitCls) {
        size_t j = i;
        uint32_t len;
        for (int m = 0; m < 3 && j < n && cls_at(j, &len) == kDigitCls; ++m) j += len;
        return j;
    }
    //  ?[^\s\p{L}\p{N}]+[\r\n]*
    {
        const size_t k = c0 == ' ' ? i + 1 : i;
        uint32_t len;
        if (k < n && cls_at(k, &len) == kOtherCls) {
            size_t j = run(k, kOtherCls);
            while (j < n && (t[j] == '\r' || t[j] == '\n')) ++j;
            return j;
        }
    }
    // a whitespace run [i, j) (kSpaceCls or kNewlineCls), `last` its last character's start
    size_t j = i, last = i, newline_end = 0;
    bool two = false;
    for (uint32_t len; j < n;) {
        const uint8_t k = cls_at(j, &len);
        if (k != kSpaceCls && k != kNewlineCls) break;
        if (k == kNewlineCls) newline_end = j + 1;
        two = j > i;
        last = j;
        j += len;
    }
    if (newline_end) return newline_end;  // \s*[\r\n]+
    if (j == n) return j;                 // \s+(?!\S) at the end of the text
    if (two) return last;                 // \s+(?!\S): all but the last character
    return j;                             // \s+
}

constexpr int kLlama3Vocab = 128256;
constexpr int kScanMax = 24;          // pieces up to this many symbols merge by array scans
constexpr size_t kCacheMaxPiece = 64;  // pieces up to this many bytes are cached
constexpr size_t kCacheMaxEntries = 1u << 16;  // per thread; cleared when full

// Piece bytes -> token ids: open addressing (linear probing, a 64-bit hash
// per slot, at most half the slots in use; the table starts at 4096 slots and
// doubles up to 2 * kCacheMaxEntries), the bytes and the ids of all entries in
// two arenas.  A slot is in use when it carries the table's current
// epoch, so emptying the table (when full, or for another tokenizer) is a new
// epoch, not a pass over the slots.
class PieceCache {
public:
    // the ids cached for p[0, n), or null; *count their number
    const int *find(const uint8_t *p, size_t n, uint64_t h, uint32_t *count) const {
        if (slots_.empty()) return nullptr;
        for (size_t i = h & mask_;; i = (i + 1) & mask_) {
            const Slot &s = slots_[i];
            if (s.epoch != epoch_) return nullptr;
            if (s.hash == h && s.key_len == n && std::memcmp(keys_.data() + s.key_off, p, n) == 0) {
                *count = s.ids_len;
                return ids_.data() + s.ids_off;
            }
        }
    }
    void insert(const uint8_t *p, size_t n, uint64_t h, const int *ids, size_t count) {
        if (slots_.empty() || entries_ >= kCacheMaxEntries) clear();
        if (2 * (entries_ + 1) > slots_.size()) grow();
        size_t i = h & mask_;
        while (slots_[i].epoch == epoch_) i = (i + 1) & mask_;
        slots_[i] = {h, static_cast<uint32_t>(keys_.size()), static_cast<uint32_t>(ids_.size()),
                     static_cast<uint16_t>(n), static_cast<uint16_t>(count), epoch_};
        keys_.insert(keys_.end(), p, p + n);
        ids_.insert(ids_.end(), ids, ids + count);
        ++entries_;
    }
    void clear() {
        if (slots_.empty() || ++epoch_ == 0) {  // first use, or the epoch counter wrapped
            slots_.assign(kFirstSlots, Slot{});
            mask_ = kFirstSlots - 1;
            epoch_ = 1;
        }
        keys_.clear();
        ids_.clear();
        entries_ = 0;
    }
    void release() {
        std::vector<Slot>().swap(slots_);
        std::vector<uint8_t>().swap(keys_);
        std::vector<int>().swap(ids_);
        entries_ = 0;
    }
    // a 64-bit hash of the piece (8-byte words folded by multiply and shift)
    static uint64_t hash(const uint8_t *p, size_t n) {
        uint64_t h = 0x9e3779b97f4a7c15ull ^ (n * 0xff51afd7ed558ccdull);
        size_t k = 0;
        for (; k + 8 <= n; k += 8) {
            uint64_t w;
            std::memcpy(&w, p + k, 8);
            h = (h ^ w) * 0xc4ceb9fe1a85ec53ull;
            h ^= h >> 31;
        }
        uint64_t w = 0;
        std::memcpy(&w, p + k, n - k);
        h = (h ^ w) * 0xc4ceb9fe1a85ec53ull;
        h ^= h >> 29;
        return h;
    }

private:
    static constexpr size_t kFirstSlots = 4096;
    void grow() {  // twice the slots, the current entries placed again
        std::vector<Slot> old(2 * slots_.size(), Slot{});
        old.swap(slots_);
        mask_ = slots_.size() - 1;
        for (const Slot &s : old) {
            if (s.epoch != epoch_) continue;
            size_t i = s.hash & mask_;
            while (slots_[i].epoch == epoch_) i = (i + 1) & mask_;
            slots_[i] = s;
        }
    }
    struct Slot {
        uint64_t hash;
        uint32_t key_off, ids_off;
        uint16_t key_len, ids_len;
        uint32_t epoch;  // 0: never used
    };
    std::vector<Slot> slots_;
    std::vector<uint8_t> keys_;
    std::vector<int> ids_;
    size_t mask_ = 0, entries_ = 0;
    uint32_t epoch_ = 1;
};
// Each thread's piece cache, tagged with the generation of the tokenizer that
// filled it (generations are never reused, so a cache is never read for
// another tokenizer); using another tokenizer on the thread clears it.
std::atomic<uint64_t> g_tokenizer_generation{0};
struct ThreadCache {
    uint64_t generation = 0;
    PieceCache map;
};
thread_local ThreadCache t_cache;

}  // namespace

struct ijb_tokenizer {
    std::vector<std::string> tokens;
    std::unordered_map<std::string, int> ids;            // first occurrence of a token string
    std::unordered_map<std::string, int> rank;           // first occurrence of a merge string
    std::unordered_map<uint64_t, uint64_t> pair;         // (left id, right id) -> rank << 32 | merged id
    // the same map frozen for lookups: open addressing over 2^pair_bits slots
    // (Fibonacci hashing, linear probing, key ~0 = empty)
    std::vector<uint64_t> pair_keys, pair_vals;
    int pair_bits = 0;
    int byte_id[256];                                    // token id of each byte's symbol
    std::string byte_symbol[256];
    std::unordered_map<std::string, uint8_t> symbol_byte;
    bool regular = true;  // every byte symbol and every merge result is a token: the id fast path applies
    std::vector<std::string> decoded;  // bytes of each token
    std::vector<uint8_t> decode_err;   // 0, 1 malformed UTF-8, 2 a character that is no byte symbol
    void *code = nullptr;
    bool jit = false;
    const uint8_t *classes = nullptr;  // code point classes for scan_piece; null: PCRE2 matches every piece
    const uint64_t generation = ++g_tokenizer_generation;
    std::string error;

    ~ijb_tokenizer() {
        if (code) pcre2().code_free(code);
        if (t_cache.generation == generation) {  // this thread's cache memory goes now
            t_cache.map.release();
            t_cache.generation = 0;
        }
    }

    // ------------------------------------------------------- BPE, by ids --
    uint64_t lookup(int a, int b) const {
        const uint64_t key = static_cast<uint64_t>(static_cast<uint32_t>(a)) << 32 | static_cast<uint32_t>(b);
        const size_t mask = pair_keys.size() - 1;
        for (size_t i = static_cast<size_t>((key * 0x9e3779b97f4a7c15ull) >> (64 - pair_bits));; i = (i + 1) & mask) {
            const uint64_t k = pair_keys[i];
            if (k == key) return pair_vals[i];
            if (k == ~0ull) return ~0ull;
        }
    }
    void freeze_pairs() {
        pair_bits = 4;
        while ((size_t{1} << pair_bits) < 2 * pair.size() + 2) ++pair_bits;
        pair_keys.assign(size_t{1} << pair_bits, ~0ull);
        pair_vals.assign(size_t{1} << pair_bits, ~0ull);
        const size_t mask = pair_keys.size() - 1;
        for (const auto &[key, val] : pair) {
            size_t i = static_cast<size_t>((key * 0x9e3779b97f4a7c15ull) >> (64 - pair_bits));
            while (pair_keys[i] != ~0ull) i = (i + 1) & mask;
            pair_keys[i] = key;
            pair_vals[i] = val;
        }
    }

    void merge_ids(const uint8_t *p, size_t n, std::vector<int> &out) const {
        if (n <= static_cast<size_t>(kScanMax)) {
            // pair[i] = (rank << 32 | merged id) of symbols i, i + 1 (~0: none);
            // a merge at `at` changes only the pairs on either side of it
            int sym[kScanMax];
            uint64_t pr[kScanMax];
            int m = static_cast<int>(n);
            for (int i = 0; i < m; ++i) sym[i] = byte_id[p[i]];
            for (int i = 0; i + 1 < m; ++i) pr[i] = lookup(sym[i], sym[i + 1]);
            while (m > 1) {
                uint64_t best = ~0ull;
                int at = -1;
                for (int i = 0; i + 1 < m; ++i)
                    if ((pr[i] >> 32) < (best >> 32)) {  // lower rank; leftmost among equals
                        best = pr[i];
                        at = i;
                    }
                if (at < 0) break;
                sym[at] = static_cast<int>(best & 0xffffffffu);
                for (int i = at + 1; i + 1 < m; ++i) sym[i] = sym[i + 1];
                for (int i = at + 1; i + 2 < m; ++i) pr[i] = pr[i + 1];
                --m;
                if (at > 0) pr[at - 1] = lookup(sym[at - 1], sym[at]);
                if (at + 1 < m) pr[at] = lookup(sym[at], sym[at + 1]);
            }
            out.insert(out.end(), sym, sym + m);
            return;
        }
        // linked symbols; heap entries (rank, left position) checked against
        // the current pair when popped (a node's id only ever grows longer)
        struct Node {
            int id, prev, next;
        };
        std::vector<Node> s(n);
        for (size_t i = 0; i < n; ++i)
            s[i] = {byte_id[p[i]], static_cast<int>(i) - 1, i + 1 < n ? static_cast<int>(i) + 1 : -1};
        struct Entry {
            uint64_t key;  // rank << 32 | left position
            int left_id, right_id;
            bool operator>(const Entry &o) const { return key > o.key; }
        };
        std::priority_queue<Entry, std::vector<Entry>, std::greater<Entry>> heap;
        auto push = [&](int i) {
            if (i < 0 || s[i].next < 0) return;
            const uint64_t v = lookup(s[i].id, s[s[i].next].id);
            if (v != ~0ull) heap.push({(v >> 32) << 32 | static_cast<uint32_t>(i), s[i].id, s[s[i].next].id});
        };
        for (size_t i = 0; i + 1 < n; ++i) push(static_cast<int>(i));
        while (!heap.empty()) {
            const Entry e = heap.top();
            heap.pop();
            const int i = static_cast<int>(e.key & 0xffffffffu);
            const int j = s[i].next;
            if (s[i].id != e.left_id || j < 0 || s[j].id != e.right_id) continue;  // stale
            s[i].id = static_cast<int>(lookup(e.left_id, e.right_id) & 0xffffffffu);
            s[i].next = s[j].next;
            if (s[j].next >= 0) s[s[j].next].prev = i;
            s[j].id = -1;
            push(s[i].prev);
            push(i);
        }
        for (int i = 0; i >= 0; i = s[i].next) out.push_back(s[i].id);
    }

    // ------------------------------------------- BPE, by strings (fallback) --
    // The merge loop on symbol strings, for vocabularies whose merges make
    // strings that are not tokens (no id to stand for them).
    void merge_strings(const uint8_t *p, size_t n, std::vector<int> &out) const {
        std::vector<std::string> parts;
        parts.reserve(n);
        for (size_t i = 0; i < n; ++i) parts.push_back(byte_symbol[p[i]]);
        while (parts.size() > 1) {
            int best = std::numeric_limits<int>::max();
            size_t at = 0;
            for (size_t i = 0; i + 1 < parts.size(); ++i) {
                const auto it = rank.find(parts[i] + " " + parts[i + 1]);
                if (it != rank.end() && it->second < best) {
                    best = it->second;
                    at = i;
                }
            }
            if (best == std::numeric_limits<int>::max()) break;
            parts[at] += parts[at + 1];
            parts.erase(parts.begin() + static_cast<long>(at) + 1);
        }
        for (const auto &s : parts) {
            const auto it = ids.find(s);
            if (it == ids.end()) throw std::runtime_error("Tokenizer produced an unknown token");
            out.push_back(it->second);
        }
    }

    // local: a piece cache the caller owns (batch workers), else this
    // thread's cache (no lock either way)
    using Cache = PieceCache;
    void piece(const uint8_t *p, size_t n, std::vector<int> &out, Cache *local) const {
        if (n == 0) return;
        if (!regular) {
            merge_strings(p, n, out);
            return;
        }
        if (n == 1) {
            out.push_back(byte_id[p[0]]);
            return;
        }
        if (n <= kCacheMaxPiece) {
            if (!local && t_cache.generation != generation) {
                t_cache.map.clear();
                t_cache.generation = generation;
            }
            Cache &c = local ? *local : t_cache.map;
            const uint64_t h = PieceCache::hash(p, n);
            uint32_t count = 0;
            if (const int *ids = c.find(p, n, h, &count)) {
                out.insert(out.end(), ids, ids + count);
                return;
            }
            const size_t first = out.size();
            merge_ids(p, n, out);
            c.insert(p, n, h, out.data() + first, out.size() - first);
            return;
        }
        merge_ids(p, n, out);
    }

    // ----------------------------------------------------- pre-tokenizer --
    void encode(const uint8_t *text, size_t n, std::vector<int> &out, Cache *local = nullptr) const {
        const Pcre2 &api = pcre2();
        // a valid text needs no UTF check per match; an invalid one is matched
        // exactly as the reference matches it (the failing call ends the loop)
        const uint32_t opts = valid_utf8(text, n) ? kPcre2NoUtfCheck : 0u;
        std::unique_ptr<void, void (*)(void *)> md(api.match_data_create(code, nullptr), api.match_data_free);
        if (!md) throw std::runtime_error("PCRE2 match data allocation failed");
        if (classes && opts == kPcre2NoUtfCheck) {  // valid UTF-8: the scanner finds every match
            for (size_t pos = 0; pos < n;) {
                const size_t e = scan_piece(text, n, pos, classes);
                piece(text + pos, e - pos, out, local);
                pos = e;
            }
            return;
        }
        size_t pos = 0;
        while (pos < n) {
            const int status = api.match(code, text, n, pos, opts, md.get(), nullptr);
            if (status < 0) {
                piece(text + pos, n - pos, out, local);
                break;
            }
            const size_t *span = api.ovector(md.get());
            if (span[0] > pos) piece(text + pos, span[0] - pos, out, local);
            if (span[1] == span[0]) throw std::runtime_error("Tokenizer regex made no progress");
            piece(text + span[0], span[1] - span[0], out, local);
            pos = span[1];
        }
    }
};

namespace {

void build(ijb_tokenizer &t, const char *const *tokens, int n_tokens, const char *const *merges, int n_merges) {
    if (n_tokens != kLlama3Vocab) throw std::runtime_error("Expected Llama 3 tokenizer");
    t.tokens.reserve(n_tokens);
    t.ids.reserve(n_tokens);
    for (int i = 0; i < n_tokens; ++i) {
        if (!tokens[i]) throw std::runtime_error("null token string");
        t.tokens.emplace_back(tokens[i]);
        t.ids.emplace(t.tokens.back(), i);
    }
    t.rank.reserve(n_merges);
    for (int i = 0; i < n_merges; ++i) {
        if (!merges[i]) throw std::runtime_error("null merge string");
        t.rank.emplace(merges[i], i);
    }
    uint32_t cp = 256;
    for (int b = 0; b < 256; ++b) {
        const bool plain = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || b >= 174;
        t.byte_symbol[b] = utf8_of(plain ? static_cast<uint32_t>(b) : cp++);
        t.symbol_byte.emplace(t.byte_symbol[b], static_cast<uint8_t>(b));
        const auto it = t.ids.find(t.byte_symbol[b]);
        t.byte_id[b] = it == t.ids.end() ? -1 : it->second;
        if (t.byte_id[b] < 0) t.regular = false;
    }
    // merges as id pairs: "A B" applies where a part A meets a part B; with
    // every result a token, each part is always a token (by induction from
    // the byte symbols), so the pair map covers every merge that can apply
    t.pair.reserve(static_cast<size_t>(n_merges) * 2);
    for (const auto &[m, r] : t.rank) {
        for (size_t sp = m.find(' '); sp != std::string::npos; sp = m.find(' ', sp + 1)) {
            const auto a = t.ids.find(m.substr(0, sp)), b = t.ids.find(m.substr(sp + 1));
            if (a == t.ids.end() || b == t.ids.end()) continue;
            const auto ab = t.ids.find(a->first + b->first);
            if (ab == t.ids.end()) {
                t.regular = false;  // a merge whose result is no token
                continue;
            }
            const uint64_t key = static_cast<uint64_t>(static_cast<uint32_t>(a->second)) << 32 |
                                 static_cast<uint32_t>(b->second);
            const uint64_t val = static_cast<uint64_t>(static_cast<uint32_t>(r)) << 32 |
                                 static_cast<uint32_t>(ab->second);
            const auto ins = t.pair.emplace(key, val);
            if (!ins.second && (val >> 32) < (ins.first->second >> 32)) ins.first->second = val;
        }
    }
    t.freeze_pairs();
    // decode table: each UTF-8 character of a token string is one byte symbol
    // (lead-byte lengths as inferencer.cu:434-441 reads them)
    t.decoded.resize(n_tokens);
    t.decode_err.assign(n_tokens, 0);
    for (int id = 0; id < n_tokens; ++id) {
        const std::string &s = t.tokens[id];
        std::string bytes;
        for (size_t i = 0; i < s.size();) {
            const uint8_t first = static_cast<uint8_t>(s[i]);
            const size_t n = first < 0x80 ? 1 : first < 0xe0 ? 2 : first < 0xf0 ? 3 : 4;
            if (i + n > s.size()) {
                t.decode_err[id] = 1;
                break;
            }
            const auto it = t.symbol_byte.find(s.substr(i, n));
            if (it == t.symbol_byte.end()) {
                t.decode_err[id] = 2;
                break;
            }
            bytes.push_back(static_cast<char>(it->second));
            i += n;
        }
        t.decoded[id] = std::move(bytes);
    }
    const Pcre2 &api = pcre2();
    int err = 0;
    size_t off = 0;
    t.code = api.compile(reinterpret_cast<const uint8_t *>(kPattern), kPcre2ZeroTerminated, kPcre2Utf | kPcre2Ucp, &err,
                         &off, nullptr);
    if (!t.code) throw std::runtime_error("Could not compile tokenizer regex");
    t.jit = api.jit_compile && api.jit_compile(t.code, kPcre2JitComplete) == 0;
    const char *env = std::getenv("IJB_TOKENIZER_SCAN");  // diagnostic: 0 = PCRE2 for every match
    if (!(env && std::atoi(env) == 0)) {
        const std::vector<uint8_t> *cls = code_point_classes();
        t.classes = cls ? cls->data() : nullptr;
    }
}

thread_local std::string t_create_err;  // message of the last failed ijb_tokenizer_create in this thread

int fail(ijb_tokenizer *t, const std::exception &e) {
    t->error = e.what();
    return IJB_ERR_INVALID;
}

}  // namespace

extern "C" {

int ijb_tokenizer_create(const char *const *tokens, int n_tokens, const char *const *merges, int n_merges,
                         ijb_tokenizer **out) {
    t_create_err.clear();
    if (!out) {
        t_create_err = "bad arguments";
        return IJB_ERR_INVALID;
    }
    *out = nullptr;
    try {
        if ((n_tokens > 0 && !tokens) || n_tokens < 0 || (n_merges > 0 && !merges) || n_merges < 0)
            throw std::runtime_error("bad arguments");
        std::unique_ptr<ijb_tokenizer> t(new ijb_tokenizer());
        build(*t, tokens, n_tokens, merges, n_merges);
        *out = t.release();
        return IJB_OK;
    } catch (const std::bad_alloc &) {
        t_create_err = "host allocation failed";
        return IJB_ERR_NOMEM;
    } catch (const std::exception &e) {
        t_create_err = e.what();
        return IJB_ERR_INVALID;
    }
}

void ijb_tokenizer_destroy(ijb_tokenizer *t) { delete t; }

const char *ijb_tokenizer_last_error(const ijb_tokenizer *t) { return t ? t->error.c_str() : t_create_err.c_str(); }

int ijb_tokenizer_encode(ijb_tokenizer *t, const char *text, long len, int *ids, long cap, long *n) {
    if (!t) return IJB_ERR_INVALID;
    try {
        if (!n || len < 0 || (len > 0 && !text) || cap < 0 || (cap > 0 && !ids)) throw std::runtime_error("bad arguments");
        if (!t->code) throw std::runtime_error("tokenizer was not created");
        std::vector<int> out;
        out.reserve(static_cast<size_t>(len) / 3 + 8);
        t->encode(reinterpret_cast<const uint8_t *>(text), static_cast<size_t>(len), out);
        *n = static_cast<long>(out.size());
        std::memcpy(ids, out.data(), std::min(out.size(), static_cast<size_t>(cap)) * sizeof(int));
        return IJB_OK;
    } catch (const std::exception &e) {
        return fail(t, e);
    }
}

int ijb_tokenizer_decode(ijb_tokenizer *t, int id, char *bytes, int cap, int *len) {
    if (!t) return IJB_ERR_INVALID;
    try {
        if (!len || cap < 0 || (cap > 0 && !bytes)) throw std::runtime_error("bad arguments");
        if (id < 0 || id >= static_cast<int>(t->tokens.size())) throw std::runtime_error("Invalid token id");
        if (t->decode_err[id] == 1) throw std::runtime_error("Malformed token UTF-8");
        if (t->decode_err[id] == 2) throw std::runtime_error("Cannot decode token");
        const std::string &s = t->decoded[id];
        *len = static_cast<int>(s.size());
        std::memcpy(bytes, s.data(), std::min(s.size(), static_cast<size_t>(cap)));
        return IJB_OK;
    } catch (const std::exception &e) {
        return fail(t, e);
    }
}

int ijb_tokenizer_special(ijb_tokenizer *t, const char *name, int *id) {
    if (!t) return IJB_ERR_INVALID;
    try {
        if (!name || !id) throw std::runtime_error("bad arguments");
        const auto it = t->ids.find(name);
        if (it == t->ids.end()) throw std::runtime_error(std::string("Missing special token ") + name);
        *id = it->second;
        return IJB_OK;
    } catch (const std::exception &e) {
        return fail(t, e);
    }
}

// Many texts at once on `threads` host threads (0: the hardware's), texts
// taken in turn from a shared counter, each worker with its own piece cache.
int ijb_tokenizer_encode_batch(ijb_tokenizer *t, const char *const *texts, const long *lens, int n_texts, int *ids,
                               long cap, long *offsets, int threads) {
    if (!t) return IJB_ERR_INVALID;
    try {
        if (n_texts < 0 || (n_texts > 0 && (!texts || !lens)) || !offsets || cap < 0 || (cap > 0 && !ids) ||
            threads < 0)
            throw std::runtime_error("bad arguments");
        if (!t->code) throw std::runtime_error("tokenizer was not created");
        for (int i = 0; i < n_texts; ++i)
            if (lens[i] < 0 || (lens[i] > 0 && !texts[i])) throw std::runtime_error("bad arguments");
        std::vector<std::vector<int>> out(static_cast<size_t>(n_texts));
        int nt = threads ? threads : static_cast<int>(std::thread::hardware_concurrency());
        nt = std::max(1, std::min(nt, n_texts));
        std::atomic<int> next{0};
        std::mutex err_mu;
        std::string err;
        auto work = [&] {
            ijb_tokenizer::Cache local;
            for (int i = next++; i < n_texts; i = next++) {
                try {
                    t->encode(reinterpret_cast<const uint8_t *>(texts[i]), static_cast<size_t>(lens[i]), out[i],
                              &local);
                } catch (const std::exception &e) {
                    std::lock_guard<std::mutex> lock(err_mu);
                    if (err.empty()) err = e.what();
                }
            }
        };
        std::vector<std::thread> pool;
        for (int k = 1; k < nt; ++k) pool.emplace_back(work);
        work();
        for (auto &th : pool) th.join();
        if (!err.empty()) throw std::runtime_error(err);
        long total = 0;
        for (int i = 0; i < n_texts; ++i) {
            offsets[i] = total;
            total += static_cast<long>(out[i].size());
        }
        offsets[n_texts] = total;
        if (total > cap) {
            t->error = "id buffer too small";
            return IJB_ERR_CAPACITY;
        }
        for (int i = 0; i < n_texts; ++i)
            if (!out[i].empty()) std::memcpy(ids + offsets[i], out[i].data(), out[i].size() * sizeof(int));
        return IJB_OK;
    } catch (const std::bad_alloc &) {
        t->error = "host allocation failed";
        return IJB_ERR_NOMEM;
    } catch (const std::exception &e) {
        return fail(t, e);
    }
}

// chat_prompt (inferencer.cu:1534-1551): the Llama 3 chat layout of one user
// turn followed by the assistant header.
int ijb_tokenizer_chat_prompt(ijb_tokenizer *t, const char *prompt, long len, int *ids, long cap, long *n) {
    if (!t) return IJB_ERR_INVALID;
    try {
        if (!n || len < 0 || (len > 0 && !prompt) || cap < 0 || (cap > 0 && !ids)) throw std::runtime_error("bad arguments");
        if (!t->code) throw std::runtime_error("tokenizer was not created");
        auto special = [&](const char *name) {
            const auto it = t->ids.find(name);
            if (it == t->ids.end()) throw std::runtime_error(std::string("Missing special token ") + name);
            return it->second;
        };
        auto append = [&](const std::string &text, std::vector<int> &out) {
            t->encode(reinterpret_cast<const uint8_t *>(text.data()), text.size(), out);
        };
        std::vector<int> out;
        out.push_back(special("<|begin_of_text|>"));
        out.push_back(special("<|start_header_id|>"));
        append("user", out);
        out.push_back(special("<|end_header_id|>"));
        append("\n\n" + std::string(prompt ? prompt : "", static_cast<size_t>(len)), out);
        out.push_back(special("<|eot_id|>"));
        out.push_back(special("<|start_header_id|>"));
        append("assistant", out);
        out.push_back(special("<|end_header_id|>"));
        append("\n\n", out);
        *n = static_cast<long>(out.size());
        std::memcpy(ids, out.data(), std::min(out.size(), static_cast<size_t>(cap)) * sizeof(int));
        return IJB_OK;
    } catch (const std::exception &e) {
        return fail(t, e);
    }
}

}  // extern "C"
