// C++ shim with the reference tokenizer's class name, constructor and method
// signatures over the C ABI (ijb_tokenizer_* in include/ijb200.h).
//
// The reference's host code builds `Tokenizer tok(model)` from its GGUF
// (inferencer.cu:368), then calls tok.encode(text) (:415), tok.decode(id)
// (:432) and tok.special(name) (:446), directly and through chat_prompt
// (:1534-1551).  This header keeps those names and argument meanings, so that
// code compiles against it unchanged once it includes this header instead of
// defining its own Tokenizer (namespace ijb_host; `using ijb_host::Tokenizer;`).
// Failures are rethrown as std::runtime_error with the reference's messages.
//
// Header-only; link libijb200.so (no GPU is touched).  The GGUF type is a
// template parameter: anything with the reference GGUF's `tokens` and
// `merges` string vectors (inferencer.cu:207) works.
#pragma once

#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/ijb200.h"

namespace ijb_host {

class Tokenizer {
public:
    template <class GGUFT>
    explicit Tokenizer(const GGUFT &model) {
        std::vector<const char *> toks, merges;
        toks.reserve(model.tokens.size());
        for (const auto &t : model.tokens) toks.push_back(t.c_str());
        merges.reserve(model.merges.size());
        for (const auto &m : model.merges) merges.push_back(m.c_str());
        if (ijb_tokenizer_create(toks.data(), static_cast<int>(toks.size()), merges.data(),
                                 static_cast<int>(merges.size()), &t_) != IJB_OK)
            throw std::runtime_error(ijb_tokenizer_last_error(nullptr));
    }
    ~Tokenizer() { ijb_tokenizer_destroy(t_); }
    Tokenizer(const Tokenizer &) = delete;
    Tokenizer &operator=(const Tokenizer &) = delete;

    std::vector<int> encode(const std::string &text) const {
        std::vector<int> out(text.size() + 16);
        long n = 0;
        check(ijb_tokenizer_encode(t_, text.data(), static_cast<long>(text.size()), out.data(),
                                   static_cast<long>(out.size()), &n));
        if (n > static_cast<long>(out.size())) {
            out.resize(static_cast<size_t>(n));
            check(ijb_tokenizer_encode(t_, text.data(), static_cast<long>(text.size()), out.data(), n, &n));
        }
        out.resize(static_cast<size_t>(n));
        return out;
    }
    std::string decode(int id) const {
        std::string s(64, '\0');
        int len = 0;
        check(ijb_tokenizer_decode(t_, id, &s[0], static_cast<int>(s.size()), &len));
        if (len > static_cast<int>(s.size())) {
            s.resize(static_cast<size_t>(len));
            check(ijb_tokenizer_decode(t_, id, &s[0], len, &len));
        }
        s.resize(static_cast<size_t>(len));
        return s;
    }
    int special(const std::string &name) const {
        int id = -1;
        check(ijb_tokenizer_special(t_, name.c_str(), &id));
        return id;
    }

private:
    void check(int rc) const {
        if (rc != IJB_OK) throw std::runtime_error(ijb_tokenizer_last_error(t_));
    }
    ijb_tokenizer *t_ = nullptr;
};

}  // namespace ijb_host
