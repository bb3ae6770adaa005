// The SentencePiece tokenizer a GGUF file carries, and the chat step API of
// the reference's Android front-end, over a GGUF session.
//
// Tokenizer: the semantics of examples/llm/model/tokenizer.cpp (encode,
// decode, decode_one). CONTROL and UNKNOWN tokens are cut out of the text
// first (longest spelling wins); each remaining fragment gets a leading space
// marker (add_space_prefix), spaces become U+2581, and adjacent symbols are
// merged best-score-first (ties: leftmost pair) while the merged spelling is
// in the vocabulary; characters left without a token fall back to one
// "<0xAB>" byte token per UTF-8 byte (or unknown). Decoding turns U+2581 back
// into spaces, resolves byte tokens, and drops one leading space.
//
// Chat: android/app/src/main/cpp/llm_jni.cpp:59-186 (create, prefill in the
// Gemma turn template with BOS on the first turn only, step one piece at a
// time until <end_of_turn> or EOS, metrics, reset).
#pragma once
#include <chrono>
#include <cstdio>
#include <queue>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

#include "gguf_model.cuh"

namespace xp {

enum : int32_t { TOK_NORMAL = 1, TOK_UNKNOWN = 2, TOK_CONTROL = 3, TOK_USER = 4, TOK_UNUSED = 5, TOK_BYTE = 6 };

class Tokenizer {
   public:
    int32_t bos = -1, eos = -1, unk = -1, pad = -1;
    bool add_bos = true, add_eos = false, space_prefix = true;
    std::string model = "llama";

    xp_status load(const GgufFile& f) {
        auto tk = f.kv.find("tokenizer.ggml.tokens");
        if (tk == f.kv.end() || tk->second.type != 9 || tk->second.elem_type != 8)
            return fail(XP_ERR_INVALID, "tokenizer: tokenizer.ggml.tokens missing or not a string array");
        vocab_ = tk->second.strs;
        const size_t n = vocab_.size();
        score_.assign(n, 0.0f);
        kind_.assign(n, TOK_NORMAL);
        if (auto sc = f.kv.find("tokenizer.ggml.scores"); sc != f.kv.end()) {
            if (sc->second.nums.size() != n) return fail(XP_ERR_INVALID, "tokenizer: scores and tokens differ in length");
            for (size_t i = 0; i < n; ++i) score_[i] = (float)sc->second.nums[i];
        }
        if (auto ty = f.kv.find("tokenizer.ggml.token_type"); ty != f.kv.end()) {
            if (ty->second.nums.size() != n)
                return fail(XP_ERR_INVALID, "tokenizer: token_type and tokens differ in length");
            for (size_t i = 0; i < n; ++i) kind_[i] = (int32_t)ty->second.nums[i];
        }
        if (std::string m = f.get_s("tokenizer.ggml.model"); !m.empty()) model = m;
        auto id = [&](const char* k, int32_t& dst) {
            uint64_t v;
            if (f.get_u(k, v)) dst = (int32_t)v;
        };
        id("tokenizer.ggml.bos_token_id", bos);
        id("tokenizer.ggml.eos_token_id", eos);
        id("tokenizer.ggml.unknown_token_id", unk);
        id("tokenizer.ggml.padding_token_id", pad);
        auto flag = [&](const char* k, bool& dst) {
            uint64_t v;
            if (f.get_u(k, v)) dst = v != 0;
        };
        flag("tokenizer.ggml.add_bos_token", add_bos);
        flag("tokenizer.ggml.add_eos_token", add_eos);
        flag("tokenizer.ggml.add_space_prefix", space_prefix);
        index_.reserve(n * 2);
        for (int32_t& b : byte_id_) b = -1;
        std::vector<size_t> lens;
        for (size_t i = 0; i < n; ++i) {
            index_.emplace(vocab_[i], (int32_t)i);  // the lowest id keeps a duplicated spelling
            if (is_special(kind_[i]) && !vocab_[i].empty()) lens.push_back(vocab_[i].size());
            int v;
            if (kind_[i] == TOK_BYTE && byte_value(vocab_[i], v)) byte_id_[v] = (int32_t)i;
        }
        std::sort(lens.begin(), lens.end(), std::greater<size_t>());
        lens.erase(std::unique(lens.begin(), lens.end()), lens.end());
        special_len_ = lens;
        return XP_OK;
    }

    size_t size() const { return vocab_.size(); }
    const std::string& text(int32_t id) const {
        static const std::string none;
        return id >= 0 && (size_t)id < vocab_.size() ? vocab_[id] : none;
    }
    int32_t kind(int32_t id) const { return id >= 0 && (size_t)id < kind_.size() ? kind_[id] : 0; }

    std::vector<int32_t> encode(std::string_view s, bool with_bos, bool with_eos) const {
        std::vector<int32_t> out;
        if (with_bos && bos >= 0) out.push_back(bos);
        size_t frag = 0;
        for (size_t i = 0; i < s.size();) {
            const int32_t hit = special_at(s, i);
            if (hit < 0) {
                ++i;
                continue;
            }
            segment(s.substr(frag, i - frag), out);
            out.push_back(hit);
            i += vocab_[hit].size();
            frag = i;
        }
        segment(s.substr(frag), out);
        if (with_eos && eos >= 0) out.push_back(eos);
        return out;
    }

    // one token's text: byte tokens as their byte, U+2581 as a space
    std::string piece(int32_t id) const {
        const std::string& t = text(id);
        int v;
        if (kind(id) == TOK_BYTE) return byte_value(t, v) ? std::string(1, (char)v) : t;
        std::string out;
        out.reserve(t.size());
        for (size_t i = 0; i < t.size();) {
            if (t.compare(i, 3, kMarker) == 0) {
                out += ' ';
                i += 3;
            } else {
                out += t[i++];
            }
        }
        return out;
    }

    std::string decode(const int32_t* ids, size_t n, bool skip_special) const {
        std::string out;
        bool first = true;
        for (size_t k = 0; k < n; ++k) {
            const bool special = is_special(kind(ids[k]));
            if (skip_special && special) continue;
            std::string p = piece(ids[k]);
            if (first && space_prefix && !p.empty() && p[0] == ' ') p.erase(0, 1);
            if (!special) first = false;
            out += p;
        }
        return out;
    }

   private:
    static constexpr const char* kMarker = "\xe2\x96\x81";  // U+2581
    std::vector<std::string> vocab_;
    std::vector<float> score_;
    std::vector<int32_t> kind_;
    std::unordered_map<std::string, int32_t> index_;
    std::vector<size_t> special_len_;  // distinct lengths of CONTROL/UNKNOWN spellings, longest first
    int32_t byte_id_[256];

    static bool is_special(int32_t k) { return k == TOK_CONTROL || k == TOK_UNKNOWN; }
    static int hexval(char c) {
        if (c >= '0' && c <= '9') return c - '0';
        if (c >= 'a' && c <= 'f') return c - 'a' + 10;
        if (c >= 'A' && c <= 'F') return c - 'A' + 10;
        return -1;
    }
    // "<0xAB>" -> 0xAB
    static bool byte_value(const std::string& t, int& v) {
        if (t.size() != 6 || t.compare(0, 3, "<0x") || t[5] != '>') return false;
        const int hi = hexval(t[3]), lo = hexval(t[4]);
        if (hi < 0) return false;
        v = lo < 0 ? hi : hi * 16 + lo;
        return true;
    }
    int32_t lookup(std::string_view s) const {
        auto it = index_.find(std::string(s));
        return it == index_.end() ? -1 : it->second;
    }
    int32_t special_at(std::string_view s, size_t i) const {
        for (size_t len : special_len_) {
            if (len > s.size() - i) continue;
            const int32_t id = lookup(s.substr(i, len));
            if (id >= 0 && is_special(kind_[id])) return id;
        }
        return -1;
    }
    static size_t utf8_len(unsigned char c) {
        return c < 0x80 ? 1 : (c & 0xE0) == 0xC0 ? 2 : (c & 0xF0) == 0xE0 ? 3 : (c & 0xF8) == 0xF0 ? 4 : 1;
    }

    // one run of ordinary text -> tokens (the best-score-first merge)
    void segment(std::string_view raw, std::vector<int32_t>& out) const {
        if (raw.empty()) return;
        std::string s;
        s.reserve(raw.size() + 8);
        if (space_prefix) s += kMarker;
        for (char c : raw) {
            if (c == ' ') s += kMarker;
            else s += c;
        }
        // symbols: byte ranges [off, off + len) of s, in a doubly linked list
        std::vector<size_t> off, len;
        std::vector<int> prv, nxt;
        for (size_t i = 0; i < s.size();) {
            const size_t l = std::min(utf8_len((unsigned char)s[i]), s.size() - i);
            prv.push_back((int)off.size() - 1);
            nxt.push_back(i + l == s.size() ? -1 : (int)off.size() + 1);
            off.push_back(i);
            len.push_back(l);
            i += l;
        }
        struct Cand {
            float score;
            int left;
            size_t bytes;
        };
        // max score first; among equal scores the leftmost pair
        auto later = [](const Cand& a, const Cand& b) { return a.score < b.score || (a.score == b.score && a.left > b.left); };
        std::priority_queue<Cand, std::vector<Cand>, decltype(later)> q(later);
        auto consider = [&](int a, int b) {
            if (a < 0 || b < 0) return;
            const int32_t id = lookup(std::string_view(s).substr(off[a], len[a] + len[b]));
            if (id >= 0) q.push({score_[id], a, len[a] + len[b]});
        };
        for (int i = 1; i < (int)off.size(); ++i) consider(i - 1, i);
        while (!q.empty()) {
            const Cand c = q.top();
            q.pop();
            const int a = c.left, b = nxt[a];
            // a pair that an earlier merge changed no longer applies
            if (len[a] == 0 || b < 0 || len[b] == 0 || len[a] + len[b] != c.bytes) continue;
            len[a] += len[b];
            len[b] = 0;
            nxt[a] = nxt[b];
            if (nxt[b] >= 0) prv[nxt[b]] = a;
            consider(prv[a], a);
            consider(a, nxt[a]);
        }
        for (int i = 0; i != -1; i = nxt[i]) {
            if (!len[i]) continue;
            const int32_t id = lookup(std::string_view(s).substr(off[i], len[i]));
            if (id >= 0) {
                out.push_back(id);
                continue;
            }
            for (size_t k = 0; k < len[i]; ++k) {  // byte fallback
                const int32_t b = byte_id_[(unsigned char)s[off[i] + k]];
                if (b >= 0) out.push_back(b);
                else if (unk >= 0) out.push_back(unk);
            }
        }
    }
};

}  // namespace xp

struct xp_tokenizer {
    xp::Tokenizer t;
};

// A chat over a GGUF session (llm_jni.cpp's ChatSession).
struct xp_chat {
    xp_session* s = nullptr;
    xp::Tokenizer tok;
    uint32_t eot = 0, eos = 0;
    bool done = false;
    double last_ms = 0, last_gpu_ms = 0;
};

extern "C" {

static xp_status tok_load(const char* path, xp::Tokenizer& t) {
    xp::GgufFile f;
    if (xp_status s = f.open(path); s != XP_OK) return s;
    return t.load(f);
}

xp_status xp_tokenizer_create(const char* gguf_path, xp_tokenizer** out) {
    if (!gguf_path || !out) return xp::fail(XP_ERR_INVALID, "xp_tokenizer_create: null argument");
    auto* t = new xp_tokenizer();
    if (xp_status s = tok_load(gguf_path, t->t); s != XP_OK) {
        delete t;
        return s;
    }
    *out = t;
    return XP_OK;
}
void xp_tokenizer_destroy(xp_tokenizer* t) { delete t; }

xp_status xp_tokenizer_info(const xp_tokenizer* t, uint32_t* vocab, int32_t* bos, int32_t* eos, int32_t* unk,
                            int32_t* pad) {
    if (!t) return xp::fail(XP_ERR_INVALID, "xp_tokenizer_info: null tokenizer");
    if (vocab) *vocab = (uint32_t)t->t.size();
    if (bos) *bos = t->t.bos;
    if (eos) *eos = t->t.eos;
    if (unk) *unk = t->t.unk;
    if (pad) *pad = t->t.pad;
    return XP_OK;
}

xp_status xp_tokenizer_encode(const xp_tokenizer* t, const char* text, size_t len, int add_bos, int add_eos,
                              int32_t* ids, uint32_t cap, uint32_t* n) {
    if (!t || (!text && len) || !n) return xp::fail(XP_ERR_INVALID, "xp_tokenizer_encode: null argument");
    const auto v = t->t.encode(std::string_view(text ? text : "", len), add_bos != 0, add_eos != 0);
    *n = (uint32_t)v.size();
    if (!ids) return XP_OK;
    if (cap < v.size()) return xp::fail(XP_ERR_INVALID, "xp_tokenizer_encode: %zu ids do not fit in %u", v.size(), cap);
    std::copy(v.begin(), v.end(), ids);
    return XP_OK;
}

xp_status xp_tokenizer_decode(const xp_tokenizer* t, const int32_t* ids, uint32_t n, int skip_special, char* out,
                              size_t cap, size_t* len) {
    if (!t || (!ids && n) || !len) return xp::fail(XP_ERR_INVALID, "xp_tokenizer_decode: null argument");
    const std::string s = t->t.decode(ids, n, skip_special != 0);
    *len = s.size();
    if (!out) return XP_OK;
    if (cap < s.size() + 1) return xp::fail(XP_ERR_INVALID, "xp_tokenizer_decode: %zu bytes do not fit in %zu",
                                            s.size() + 1, cap);
    std::memcpy(out, s.c_str(), s.size() + 1);
    return XP_OK;
}

xp_status xp_tokenizer_piece(const xp_tokenizer* t, int32_t id, char* out, size_t cap, size_t* len) {
    if (!t || !len) return xp::fail(XP_ERR_INVALID, "xp_tokenizer_piece: null argument");
    const std::string s = t->t.piece(id);
    *len = s.size();
    if (!out) return XP_OK;
    if (cap < s.size() + 1) return xp::fail(XP_ERR_INVALID, "xp_tokenizer_piece: buffer too small");
    std::memcpy(out, s.c_str(), s.size() + 1);
    return XP_OK;
}

xp_status xp_chat_create(int device, const char* gguf_path, uint32_t max_seq, const xp_sampling* sp,
                         const char* pack_cache, xp_chat** out) {
    if (!gguf_path || !out) return xp::fail(XP_ERR_INVALID, "xp_chat_create: null argument");
    *out = nullptr;
    // Gemma's recommended chat decoding unless the caller says otherwise
    const xp_sampling dflt{0, 0.7f, 64, 0.95f, 1234, 0};
    xp_model_config pol{};
    pol.max_seq = max_seq;
    pol.global_every = 6;
    pol.rope_theta_local = 1e4f;
    auto* c = new xp_chat();
    xp_status s = tok_load(gguf_path, c->tok);
    if (s == XP_OK) s = xp_session_create_gguf(device, gguf_path, &pol, sp ? sp : &dflt, pack_cache, &c->s);
    if (s != XP_OK) {
        delete c;
        return s;
    }
    const auto e = c->tok.encode("<end_of_turn>", false, false);
    c->eot = e.empty() ? 0u : (uint32_t)e.back();
    c->eos = c->tok.eos < 0 ? 0u : (uint32_t)c->tok.eos;
    *out = c;
    return XP_OK;
}

xp_status xp_chat_prefill(xp_chat* c, const char* text, uint32_t* n_tokens) {
    if (!c || !text) return xp::fail(XP_ERR_INVALID, "xp_chat_prefill: null argument");
    uint32_t pos = 0;
    if (xp_status s = xp_session_position(c->s, &pos); s != XP_OK) return s;
    const bool first = pos == 0;
    const std::string prompt = std::string(first ? "" : "\n") + "<start_of_turn>user\n" + text +
                               "<end_of_turn>\n<start_of_turn>model\n";
    const auto ids = c->tok.encode(prompt, first, false);
    std::vector<uint32_t> u(ids.begin(), ids.end());
    if (xp_status s = xp_session_prefill(c->s, u.data(), (uint32_t)u.size()); s != XP_OK) return s;
    c->done = false;
    if (n_tokens) *n_tokens = (uint32_t)u.size();
    return XP_OK;
}

xp_status xp_chat_step(xp_chat* c, char* piece, size_t cap, int* done) {
    if (!c || !done) return xp::fail(XP_ERR_INVALID, "xp_chat_step: null argument");
    *done = 1;
    if (piece && cap) piece[0] = 0;
    if (c->done) return XP_OK;
    const auto t0 = std::chrono::steady_clock::now();
    xp_session_timer(c->s, 0, nullptr);
    uint32_t tok = 0;
    xp_status s = xp_session_decode_step(c->s, &tok);
    float gms = 0;
    xp_session_timer(c->s, 1, &gms);
    c->last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    c->last_gpu_ms = gms;
    if (s != XP_OK) {
        c->done = true;
        return s;
    }
    if (tok == c->eot || tok == c->eos) {
        c->done = true;
        return XP_OK;
    }
    uint32_t pos = 0;
    xp_session_position(c->s, &pos);
    if (pos + 1 >= c->s->cfg.max_seq) c->done = true;  // the next turn must not run out of KV rows
    const std::string p = c->tok.piece((int32_t)tok);
    if (piece) {
        if (cap < p.size() + 1) return xp::fail(XP_ERR_INVALID, "xp_chat_step: piece buffer too small");
        std::memcpy(piece, p.c_str(), p.size() + 1);
    }
    *done = 0;
    return XP_OK;
}

// {ms, tok/s, kernels, submits, position, record_ms, gpu_ms} of the last step
xp_status xp_chat_metrics(const xp_chat* c, double out[7]) {
    if (!c || !out) return xp::fail(XP_ERR_INVALID, "xp_chat_metrics: null argument");
    uint32_t pos = 0;
    xp_session_position(c->s, &pos);
    out[0] = c->last_ms;
    out[1] = c->last_ms > 0 ? 1000.0 / c->last_ms : 0.0;
    out[2] = c->s->kernels_per_token;
    out[3] = 1;  // one graph launch per step
    out[4] = pos;
    out[5] = 0;  // nothing is recorded per step: the graph is replayed
    out[6] = c->last_gpu_ms;
    return XP_OK;
}

xp_status xp_chat_session(xp_chat* c, xp_session** s) {
    if (!c || !s) return xp::fail(XP_ERR_INVALID, "xp_chat_session: null argument");
    *s = c->s;
    return XP_OK;
}

xp_status xp_chat_reset(xp_chat* c) {
    if (!c) return xp::fail(XP_ERR_INVALID, "xp_chat_reset: null chat");
    c->done = false;
    return xp_session_reset(c->s);
}

void xp_chat_destroy(xp_chat* c) {
    if (!c) return;
    if (c->s) xp_session_destroy(c->s);
    delete c;
}

}  // extern "C"
