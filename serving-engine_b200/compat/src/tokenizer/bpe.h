// compat/src/tokenizer/bpe.h -- the reference's engine::BPETokenizer and
// ChatMessage (src/tokenizer/bpe.h:10-58) over the b2engine tokenizer
// (b2_tokenizer_*).  Public interface, defaults and failure behaviour as in
// the reference: load() returns false with a message on stderr; encode,
// decode and apply_chat_template keep their signatures; the three control-
// token accessors fall back to the Qwen2 ids when the vocabulary lacks them.
//
// Behaviour beyond the reference, all of it the HF tokenizers library's:
// Llama-3 and GPT-2 vocabularies load as well as Qwen2 ones; the file's NFC
// normaliser is applied; encode(text, false) reads only the tokens marked
// special as text (non-special added tokens are still split out), and
// decode(ids, true) drops only special tokens; apply_chat_template writes the
// Llama-3 format for a Llama-3 vocabulary.
#pragma once

#include <cstdint>
#include <iostream>
#include <memory>
#include <string>
#include <vector>

#include "src/b2_compat.h"

namespace engine {

struct ChatMessage {
    std::string role;
    std::string content;
};

class BPETokenizer {
public:
    BPETokenizer() = default;
    ~BPETokenizer() = default;

    // Load from HF tokenizer.json
    bool load(const std::string& tokenizer_json_path) {
        b2_tokenizer* t = nullptr;
        int rc = b2_tokenizer_load(tokenizer_json_path.c_str(), &t);
        if (rc != 0) {
            std::cerr << "Failed to load tokenizer.json: " << tokenizer_json_path << " (" << b2_status_string(rc)
                      << ": " << b2_last_error() << ")" << std::endl;
            return false;
        }
        t_.reset(t, b2_tokenizer_destroy);
        b2_tokenizer_info info;
        cuda::b2_check(b2_tokenizer_get_info(t, &info), "BPETokenizer::load");
        vocab_size_ = (size_t)info.vocab_size;
        im_start_id_ = id_or(t, "<|im_start|>", 151644);
        im_end_id_ = id_or(t, "<|im_end|>", 151645);
        endoftext_id_ = id_or(t, "<|endoftext|>", 151643);
        return true;
    }

    // Encode text to token IDs
    std::vector<int> encode(const std::string& text, bool allowed_special = true) const {
        std::vector<int> ids(text.size() + 8);
        size_t n = 0;
        const int flags = allowed_special ? B2_TOK_SPLIT_SPECIAL : 0;
        int rc = b2_tokenizer_encode(tok(), text.data(), text.size(), flags, reinterpret_cast<int32_t*>(ids.data()),
                                     ids.size(), &n);
        if (rc == B2_ERR_WORKSPACE) {
            ids.resize(n);
            rc = b2_tokenizer_encode(tok(), text.data(), text.size(), flags, reinterpret_cast<int32_t*>(ids.data()),
                                     ids.size(), &n);
        }
        cuda::b2_check(rc, "BPETokenizer::encode");
        ids.resize(n);
        return ids;
    }

    // Decode token IDs back to UTF-8 text
    std::string decode(const std::vector<int>& ids, bool skip_special_tokens = false) const {
        std::string out(ids.size() * 8 + 16, '\0');
        size_t n = 0;
        const int32_t* p = reinterpret_cast<const int32_t*>(ids.data());
        int rc = b2_tokenizer_decode(tok(), p, ids.size(), skip_special_tokens, &out[0], out.size(), &n);
        if (rc == B2_ERR_WORKSPACE) {
            out.resize(n);
            rc = b2_tokenizer_decode(tok(), p, ids.size(), skip_special_tokens, &out[0], out.size(), &n);
        }
        cuda::b2_check(rc, "BPETokenizer::decode");
        out.resize(n);
        return out;
    }

    // Apply the vocabulary's chat template (Qwen ChatML, or Llama-3)
    std::string apply_chat_template(const std::vector<ChatMessage>& messages, bool add_generation_prompt = true) const {
        std::vector<const char*> roles, contents;
        size_t total = 256;
        for (const auto& m : messages) {
            roles.push_back(m.role.c_str());
            contents.push_back(m.content.c_str());
            total += m.role.size() + m.content.size() + 64;
        }
        std::string out(total, '\0');
        size_t n = 0;
        int rc = b2_tokenizer_apply_chat_template(tok(), roles.data(), contents.data(), messages.size(),
                                                  add_generation_prompt, &out[0], out.size(), &n);
        if (rc == B2_ERR_WORKSPACE) {
            out.resize(n);
            rc = b2_tokenizer_apply_chat_template(tok(), roles.data(), contents.data(), messages.size(),
                                                  add_generation_prompt, &out[0], out.size(), &n);
        }
        cuda::b2_check(rc, "BPETokenizer::apply_chat_template");
        out.resize(n);
        return out;
    }

    // Special token IDs
    int im_start_id() const { return im_start_id_; }
    int im_end_id() const { return im_end_id_; }
    int endoftext_id() const { return endoftext_id_; }

    size_t vocab_size() const { return vocab_size_; }

private:
    const b2_tokenizer* tok() const {
        if (!t_) throw std::runtime_error("BPETokenizer used before load()");
        return t_.get();
    }
    static int id_or(const b2_tokenizer* t, const char* s, int fallback) {
        int32_t id = -1;
        return b2_tokenizer_token_to_id(t, s, std::char_traits<char>::length(s), &id) == 0 ? id : fallback;
    }

    std::shared_ptr<b2_tokenizer> t_;
    size_t vocab_size_ = 0;
    int im_start_id_ = 151644;
    int im_end_id_ = 151645;
    int endoftext_id_ = 151643;
};

}  // namespace engine
