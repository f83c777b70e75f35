// chatdata.cpp -- chat JSONL to token ids with an assistant loss mask, as C entry points of libr97host.so.
//
// The reference's ChatData (include/r97/chatdata.h, src/chatdata.cpp) renders with the container's chat
// template and tokenizer (radiance's rad_core, not in this tree) and adds the loss mask; this file keeps the
// same split. The renderer is an interface (ChatRenderer: a conversation prefix to token ids, with or without
// the generation prompt, and which ids are control tokens); what ChatData itself decides is the reference's:
//
//   1. Keep the conversation through its last assistant turn. Render it; while the render is longer than
//      the limit, drop the last kept assistant turn (and what follows it) and render again. No assistant
//      turn left: the conversation is skipped. Dropping anything makes the outcome Shortened.
//   2. For each kept assistant turn i, the scored tokens run from the end of the render of messages [0, i)
//      with the generation prompt (what serving feeds the model before the turn) to the end of the render
//      of messages [0, i], each located as the common token prefix with the whole sequence; the span ends
//      at its last control token (the turn's end-of-turn token), so the template's separator after it is
//      not scored. A turn whose span cannot be located (stop <= start) is not scored.
//   3. A JSONL document is read line by line (blank lines skipped); each line is {"messages": [{"role":
//      string, "content": string}, ...]}; a malformed line stops the read with "line N: <why>", the lines
//      before it kept. Outcomes are counted into the stats.
//
// ChatMLByteRenderer is the stand-in renderer the tests use (the reference's own mask test builds its
// expectations the same way): Qwen's ChatML template, "<|im_start|>role\ncontent<|im_end|>\n" per message and
// "<|im_start|>assistant\n" as the generation prompt, over a byte vocabulary (ids 0-255 the bytes, 256
// <|im_start|>, 257 <|im_end|>, both control tokens, no BOS), the markers parsed as specials wherever they
// appear in the rendered text.
#include <cstdint>
#include <cstring>
#include <fstream>
#include <memory>
#include <sstream>
#include <string>
#include <string_view>
#include <vector>

namespace {

struct ChatMessage {
    std::string role, content;
};

class ChatRenderer {
public:
    virtual ~ChatRenderer() = default;
    // The first `count` messages rendered to token ids, with the generation prompt when asked.
    virtual bool render(const std::vector<ChatMessage>& messages, size_t count, bool add_generation_prompt,
                        std::vector<int32_t>* ids, std::string* error) const = 0;
    virtual bool is_control(int32_t id) const = 0;
};

class ChatMLByteRenderer : public ChatRenderer {
public:
    static constexpr int32_t kImStart = 256, kImEnd = 257;

    bool render(const std::vector<ChatMessage>& messages, size_t count, bool add_generation_prompt,
                std::vector<int32_t>* ids, std::string*) const override {
        std::string text;
        for (size_t i = 0; i < count && i < messages.size(); ++i)
            text += "<|im_start|>" + messages[i].role + "\n" + messages[i].content + "<|im_end|>\n";
        if (add_generation_prompt) text += "<|im_start|>assistant\n";
        encode(text, ids);
        return true;
    }
    bool is_control(int32_t id) const override { return id == kImStart || id == kImEnd; }

    // Bytes to ids, the two markers parsed as their special ids.
    static void encode(std::string_view text, std::vector<int32_t>* ids) {
        static constexpr std::string_view kStart = "<|im_start|>", kEnd = "<|im_end|>";
        ids->clear();
        size_t i = 0;
        while (i < text.size()) {
            if (text.compare(i, kStart.size(), kStart) == 0) {
                ids->push_back(kImStart);
                i += kStart.size();
            } else if (text.compare(i, kEnd.size(), kEnd) == 0) {
                ids->push_back(kImEnd);
                i += kEnd.size();
            } else {
                ids->push_back((int32_t)(unsigned char)text[i]);
                ++i;
            }
        }
    }
};

// ------------------------------------------------------------------------------------------ JSON
// The subset a chat line needs: objects, arrays, strings (every escape, \u with surrogate pairs, to UTF-8),
// numbers, true / false / null. Values other than the messages' strings are parsed and dropped.
struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    std::string str;
    std::vector<Json> items;                                  // Arr
    std::vector<std::pair<std::string, Json>> members;        // Obj, in order
    const Json* find(const std::string& key) const {
        for (const auto& m : members)
            if (m.first == key) return &m.second;
        return nullptr;
    }
};

class JsonReader {
public:
    explicit JsonReader(std::string_view s) : s_(s) {}
    bool document(Json* out) {
        ws();
        if (!value(out, 0)) return false;
        ws();
        return i_ == s_.size();
    }

private:
    std::string_view s_;
    size_t i_ = 0;

    void ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\t' || s_[i_] == '\n' || s_[i_] == '\r')) ++i_;
    }
    bool lit(std::string_view w) {
        if (s_.compare(i_, w.size(), w) != 0) return false;
        i_ += w.size();
        return true;
    }
    static void utf8(uint32_t cp, std::string* out) {
        if (cp < 0x80) {
            out->push_back((char)cp);
        } else if (cp < 0x800) {
            out->push_back((char)(0xC0 | (cp >> 6)));
            out->push_back((char)(0x80 | (cp & 0x3F)));
        } else if (cp < 0x10000) {
            out->push_back((char)(0xE0 | (cp >> 12)));
            out->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            out->push_back((char)(0x80 | (cp & 0x3F)));
        } else {
            out->push_back((char)(0xF0 | (cp >> 18)));
            out->push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
            out->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            out->push_back((char)(0x80 | (cp & 0x3F)));
        }
    }
    bool hex4(uint32_t* v) {
        if (i_ + 4 > s_.size()) return false;
        *v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = s_[i_++];
            *v <<= 4;
            if (c >= '0' && c <= '9') *v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') *v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') *v |= (uint32_t)(c - 'A' + 10);
            else return false;
        }
        return true;
    }
    bool string(std::string* out) {
        if (i_ >= s_.size() || s_[i_] != '"') return false;
        ++i_;
        while (i_ < s_.size()) {
            const char c = s_[i_++];
            if (c == '"') return true;
            if ((unsigned char)c < 0x20) return false;
            if (c != '\\') {
                out->push_back(c);
                continue;
            }
            if (i_ >= s_.size()) return false;
            const char e = s_[i_++];
            switch (e) {
                case '"': out->push_back('"'); break;
                case '\\': out->push_back('\\'); break;
                case '/': out->push_back('/'); break;
                case 'b': out->push_back('\b'); break;
                case 'f': out->push_back('\f'); break;
                case 'n': out->push_back('\n'); break;
                case 'r': out->push_back('\r'); break;
                case 't': out->push_back('\t'); break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(&cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {  // a high surrogate: its low half must follow
                        uint32_t lo;
                        if (!lit("\\u") || !hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return false;
                    }
                    utf8(cp, out);
                    break;
                }
                default: return false;
            }
        }
        return false;
    }
    bool number() {
        const size_t b = i_;
        if (i_ < s_.size() && s_[i_] == '-') ++i_;
        size_t d = 0;
        while (i_ < s_.size() && s_[i_] >= '0' && s_[i_] <= '9') ++i_, ++d;
        if (d == 0) return false;
        if (i_ < s_.size() && s_[i_] == '.') {
            ++i_;
            d = 0;
            while (i_ < s_.size() && s_[i_] >= '0' && s_[i_] <= '9') ++i_, ++d;
            if (d == 0) return false;
        }
        if (i_ < s_.size() && (s_[i_] == 'e' || s_[i_] == 'E')) {
            ++i_;
            if (i_ < s_.size() && (s_[i_] == '+' || s_[i_] == '-')) ++i_;
            d = 0;
            while (i_ < s_.size() && s_[i_] >= '0' && s_[i_] <= '9') ++i_, ++d;
            if (d == 0) return false;
        }
        return i_ > b;
    }
    bool value(Json* out, int depth) {
        if (depth > 64 || i_ >= s_.size()) return false;
        const char c = s_[i_];
        if (c == '{') {
            out->kind = Json::Obj;
            ++i_;
            ws();
            if (i_ < s_.size() && s_[i_] == '}') return ++i_, true;
            while (true) {
                ws();
                std::string key;
                if (!string(&key)) return false;
                ws();
                if (i_ >= s_.size() || s_[i_] != ':') return false;
                ++i_;
                ws();
                Json v;
                if (!value(&v, depth + 1)) return false;
                out->members.emplace_back(std::move(key), std::move(v));
                ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    ++i_;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == '}') return ++i_, true;
                return false;
            }
        }
        if (c == '[') {
            out->kind = Json::Arr;
            ++i_;
            ws();
            if (i_ < s_.size() && s_[i_] == ']') return ++i_, true;
            while (true) {
                ws();
                Json v;
                if (!value(&v, depth + 1)) return false;
                out->items.push_back(std::move(v));
                ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    ++i_;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == ']') return ++i_, true;
                return false;
            }
        }
        if (c == '"') {
            out->kind = Json::Str;
            return string(&out->str);
        }
        if (lit("true") || lit("false")) return out->kind = Json::Bool, true;
        if (lit("null")) return out->kind = Json::Null, true;
        out->kind = Json::Num;
        return number();
    }
};

// ------------------------------------------------------------------------------------------ ChatData
enum Outcome { kKept = 0, kShortened = 1, kSkipped = 2, kError = 3 };

struct Stats {
    int64_t conversations, kept, shortened, skipped, tokens, scored;
};

struct Seq {
    std::vector<int32_t> ids;
    std::vector<uint8_t> score;
};

int common_prefix(const std::vector<int32_t>& a, const std::vector<int32_t>& b) {
    const size_t n = a.size() < b.size() ? a.size() : b.size();
    size_t i = 0;
    while (i < n && a[i] == b[i]) ++i;
    return (int)i;
}

class ChatData {
public:
    explicit ChatData(std::unique_ptr<ChatRenderer> r) : r_(std::move(r)) {}

    Outcome render(const std::vector<ChatMessage>& m, int max_tokens, Seq* out) {
        out->ids.clear();
        out->score.clear();
        error.clear();
        if (max_tokens <= 0) {
            error = "the token limit must be positive";
            return kError;
        }
        size_t keep = m.size();
        bool shortened = false;
        std::vector<int32_t> ids;
        while (true) {
            size_t last = keep;  // one past the last assistant turn kept
            while (last > 0 && m[last - 1].role != "assistant") --last;
            if (last == 0) return kSkipped;
            keep = last;
            if (!r_->render(m, keep, false, &ids, &error)) return kError;
            if (ids.size() <= (size_t)max_tokens) break;
            shortened = true;
            keep = last - 1;
        }
        Seq seq;
        seq.ids = ids;
        seq.score.assign(ids.size(), 0);
        std::vector<int32_t> header, turn;
        for (size_t i = 0; i < keep; ++i) {
            if (m[i].role != "assistant") continue;
            if (!r_->render(m, i, true, &header, &error)) return kError;
            if (!r_->render(m, i + 1, false, &turn, &error)) return kError;
            const int start = common_prefix(header, seq.ids);
            int stop = common_prefix(turn, seq.ids);
            if (stop <= start) continue;
            for (int j = stop - 1; j >= start; --j)
                if (r_->is_control(seq.ids[(size_t)j])) {
                    stop = j + 1;
                    break;
                }
            for (int j = start; j < stop; ++j) seq.score[(size_t)j] = 1;
        }
        *out = std::move(seq);
        return shortened ? kShortened : kKept;
    }

    Outcome line(std::string_view text, int max_tokens, Seq* out) {
        error.clear();
        Json doc;
        if (!JsonReader(text).document(&doc) || doc.kind != Json::Obj) {
            error = "the line is not a JSON object";
            return kError;
        }
        const Json* msgs = doc.find("messages");
        if (!msgs || msgs->kind != Json::Arr) {
            error = "the object has no \"messages\" array";
            return kError;
        }
        std::vector<ChatMessage> chat;
        for (const Json& j : msgs->items) {
            if (j.kind != Json::Obj) {
                error = "a message is not an object";
                return kError;
            }
            const Json* role = j.find("role");
            const Json* content = j.find("content");
            if (!role || role->kind != Json::Str) {
                error = "a message has no string \"role\"";
                return kError;
            }
            if (!content || content->kind != Json::Str) {
                error = "the \"" + role->str + "\" message has no string \"content\"";
                return kError;
            }
            chat.push_back(ChatMessage{role->str, content->str});
        }
        return render(chat, max_tokens, out);
    }

    bool read(std::string_view doc, int max_tokens, Stats* st) {
        error.clear();
        size_t pos = 0;
        int64_t line_no = 0;
        while (pos < doc.size()) {
            const size_t eol = doc.find('\n', pos);
            const std::string_view text = doc.substr(pos, eol == std::string_view::npos ? std::string_view::npos : eol - pos);
            pos = eol == std::string_view::npos ? doc.size() : eol + 1;
            ++line_no;
            if (text.find_first_not_of(" \t\r") == std::string_view::npos) continue;
            Seq seq;
            const Outcome o = line(text, max_tokens, &seq);
            if (o == kError) {
                error = "line " + std::to_string(line_no) + ": " + error;
                return false;
            }
            ++st->conversations;
            if (o == kSkipped) {
                ++st->skipped;
                continue;
            }
            ++st->kept;
            if (o == kShortened) ++st->shortened;
            st->tokens += (int64_t)seq.ids.size();
            for (uint8_t s : seq.score) st->scored += s;
            seqs.push_back(std::move(seq));
        }
        return true;
    }

    std::vector<Seq> seqs;  // the kept sequences of every read, in order
    std::string error;

private:
    std::unique_ptr<ChatRenderer> r_;
};

thread_local std::string g_chat_error;

}  // namespace

extern "C" {

// A ChatData over the ChatML byte-vocabulary renderer.
void* r97host_chatdata_create_chatml_bytes(void) {
    return new ChatData(std::make_unique<ChatMLByteRenderer>());
}

void r97host_chatdata_destroy(void* cd) { delete static_cast<ChatData*>(cd); }

// Reads a JSONL document (len bytes) and appends its kept sequences; adds its outcome counts into
// stats[6] = {conversations, kept, shortened, skipped, tokens, scored}. 1, or 0 with the reason (with its
// line number) in r97host_chatdata_error.
int32_t r97host_chatdata_read(void* cd, const char* text, int64_t len, int32_t max_tokens, int64_t* stats) {
    auto* c = static_cast<ChatData*>(cd);
    Stats st{};
    const bool ok = c->read(std::string_view(text ? text : "", text ? (size_t)len : 0), max_tokens, &st);
    if (stats) {
        stats[0] += st.conversations, stats[1] += st.kept, stats[2] += st.shortened;
        stats[3] += st.skipped, stats[4] += st.tokens, stats[5] += st.scored;
    }
    return ok ? 1 : 0;
}

// Reads a JSONL file as r97host_chatdata_read does.
int32_t r97host_chatdata_read_file(void* cd, const char* path, int32_t max_tokens, int64_t* stats) {
    auto* c = static_cast<ChatData*>(cd);
    std::ifstream f(path ? path : "", std::ios::binary);
    if (!f) {
        c->error = std::string(path ? path : "") + ": cannot read the file";
        return 0;
    }
    std::ostringstream ss;
    ss << f.rdbuf();
    const std::string s = ss.str();
    return r97host_chatdata_read(cd, s.data(), (int64_t)s.size(), max_tokens, stats);
}

// One conversation given as one JSONL line, rendered and scored without being appended: the outcome
// (0 kept, 1 shortened, 2 skipped, 3 error), and the sequence (ids, score; up to cap tokens) with its length
// in *n.
int32_t r97host_chatdata_line(void* cd, const char* text, int64_t len, int32_t max_tokens, int32_t* ids,
                              uint8_t* score, int64_t cap, int64_t* n) {
    auto* c = static_cast<ChatData*>(cd);
    Seq seq;
    const Outcome o = c->line(std::string_view(text ? text : "", text ? (size_t)len : 0), max_tokens, &seq);
    *n = (int64_t)seq.ids.size();
    for (int64_t i = 0; i < *n && i < cap; ++i) {
        ids[i] = seq.ids[(size_t)i];
        score[i] = seq.score[(size_t)i];
    }
    return (int32_t)o;
}

int64_t r97host_chatdata_count(void* cd) { return (int64_t)static_cast<ChatData*>(cd)->seqs.size(); }

int64_t r97host_chatdata_seq_len(void* cd, int64_t i) {
    const auto& v = static_cast<ChatData*>(cd)->seqs;
    return i >= 0 && (size_t)i < v.size() ? (int64_t)v[(size_t)i].ids.size() : -1;
}

// Copies sequence i's ids and score (r97host_chatdata_seq_len(i) entries each).
void r97host_chatdata_seq(void* cd, int64_t i, int32_t* ids, uint8_t* score) {
    const auto& s = static_cast<ChatData*>(cd)->seqs[(size_t)i];
    std::memcpy(ids, s.ids.data(), s.ids.size() * sizeof(int32_t));
    std::memcpy(score, s.score.data(), s.score.size());
}

const char* r97host_chatdata_error(void* cd) {
    g_chat_error = cd ? static_cast<ChatData*>(cd)->error : std::string();
    return g_chat_error.c_str();
}

}  // extern "C"
