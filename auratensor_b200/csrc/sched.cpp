// Continuous batching of generation requests over the model's KV slots.
//
// The reference serves one request at a time: the prompt token by token
// through forwardStep, then Sampler.sample -> forwardStep per generated token
// with the prompt plus the emitted tokens as the penalty history, stopping at
// maxTokens or the EOS id (server/InferenceServer.java:111-134). Here every
// active request owns one KV slot; each at_sched_step runs one batched decode
// step over slots 0..B-1 with device sampling per row. A request's prompt
// runs into its slot through the batched prompt path where the model has one
// (all but the last prompt token), otherwise token by token inside the
// batched steps, its samples discarded until the last prompt token. Rows of
// free slots below B decode a placeholder token at position 0 of their own
// slot, which the next request's prompt overwrites.
#include <deque>
#include <map>
#include <string>
#include <vector>

#include "at_internal.h"

namespace {

struct Request {
    std::vector<int> prompt;
    int max_new = 0;
    int eos = -1;
    at_sampler_config cfg{};
    std::vector<int> out;
    bool done = false;
    int slot = -1;
    int64_t pos = 0;  // tokens of this request already in its slot's KV
};

}  // namespace

struct at_sched {
    at_model* m = nullptr;
    int slots = 0;
    int64_t ctx = 0;
    int next_id = 1;
    std::map<int, Request> reqs;
    std::deque<int> waiting;
    std::vector<int> slot_req;  // request id per slot, -1 free
};

using namespace at;

namespace {

// The token a request feeds at its next position.
int next_input(const Request& r) {
    return r.pos < (int64_t)r.prompt.size() ? r.prompt[r.pos] : r.out[r.pos - r.prompt.size()];
}

void admit(at_sched* s) {
    for (int slot = 0; slot < s->slots && !s->waiting.empty(); ++slot) {
        if (s->slot_req[slot] >= 0) continue;
        const int id = s->waiting.front();
        s->waiting.pop_front();
        Request& r = s->reqs.at(id);
        r.slot = slot;
        s->slot_req[slot] = id;
        sched_reset_slot(s->m, slot);
        sched_set_row(s->m, slot, &r.cfg, r.prompt.data(), (int)r.prompt.size());
        const int prefix = (int)r.prompt.size() - 1;  // the last prompt token runs in a decode step
        if (prefix > 0 && model_slot_prompt(s->m)) {
            sched_prompt(s->m, slot, r.prompt.data(), prefix);
            r.pos = prefix;
        } else {
            r.pos = 0;
        }
    }
}

void retire(at_sched* s, Request& r) {
    r.done = true;
    s->slot_req[r.slot] = -1;
    sched_set_row(s->m, r.slot, nullptr, nullptr, 0);
    r.slot = -1;
}

}  // namespace

extern "C" {

int at_sched_create(at_model* m, at_sched** out) {
    return guard([&] {
        AT_REQUIRE(m && out, AT_ERR_INVALID_ARG, "null argument");
        auto* s = new at_sched();
        s->m = m;
        s->slots = model_max_batch(m);
        s->ctx = model_ctx_len(m);
        s->slot_req.assign(s->slots, -1);
        *out = s;
    });
}

int at_sched_destroy(at_sched* s) {
    delete s;
    return AT_OK;
}

int at_sched_submit(at_sched* s, const int* prompt, int n, int max_new, int eos_token, const at_sampler_config* cfg,
                    int* request_id) {
    return guard([&] {
        AT_REQUIRE(s && prompt && cfg && request_id, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(n >= 1, AT_ERR_INVALID_ARG, "empty prompt");
        AT_REQUIRE(max_new >= 0, AT_ERR_INVALID_ARG, "negative max_new");
        // KVCache.append (inference/KVCache.java:83-85): the reference runs
        // forwardStep after each emitted token, up to position n + max_new - 1.
        AT_REQUIRE((int64_t)n + max_new <= s->ctx, AT_ERR_INVALID_ARG,
                   "prompt of " + std::to_string(n) + " plus " + std::to_string(max_new) +
                       " tokens exceeds maxContext " + std::to_string(s->ctx));
        const int V = model_vocab(s->m);
        for (int i = 0; i < n; ++i)
            AT_REQUIRE(prompt[i] >= 0 && prompt[i] < V, AT_ERR_INVALID_ARG,
                       "token id " + std::to_string(prompt[i]) + " out of range");
        Request r;
        r.prompt.assign(prompt, prompt + n);
        r.max_new = max_new;
        r.eos = eos_token;
        r.cfg = *cfg;
        r.cfg.history = nullptr;
        r.cfg.history_len = 0;
        // the sampler settings fail here rather than at admission
        AT_REQUIRE(r.cfg.temperature == 0.0f || (r.cfg.top_k == 1 && r.cfg.top_p >= 1.0f) ||
                       (r.cfg.top_k >= 1 && std::min(r.cfg.top_k, V) <= sample_k_max()),
                   AT_ERR_UNSUPPORTED, "topK must be in 1.." + std::to_string(sample_k_max()));
        const int id = s->next_id++;
        r.done = max_new == 0;
        s->reqs.emplace(id, std::move(r));
        if (max_new > 0) s->waiting.push_back(id);
        *request_id = id;
    });
}

int at_sched_step(at_sched* s, int* n_active) {
    return guard([&] {
        AT_REQUIRE(s && n_active, AT_ERR_INVALID_ARG, "null argument");
        admit(s);
        int B = 0;
        for (int b = 0; b < s->slots; ++b)
            if (s->slot_req[b] >= 0) B = b + 1;
        if (B > 0) {
            std::vector<int> tokens(B, 0), append(B, 0), picked(B, 0);
            std::vector<int64_t> pos(B, 0);
            for (int b = 0; b < B; ++b) {
                if (s->slot_req[b] < 0) continue;
                const Request& r = s->reqs.at(s->slot_req[b]);
                tokens[b] = next_input(r);
                pos[b] = r.pos;
                append[b] = r.pos + 1 >= (int64_t)r.prompt.size();  // this step's sample is a real one
            }
            sched_step(s->m, B, tokens.data(), pos.data(), append.data(), picked.data());
            for (int b = 0; b < B; ++b) {
                if (s->slot_req[b] < 0) continue;
                Request& r = s->reqs.at(s->slot_req[b]);
                const bool real = append[b] != 0;
                r.pos += 1;
                if (!real) continue;
                const int t = picked[b];
                if (t == r.eos) {
                    retire(s, r);
                    continue;
                }
                r.out.push_back(t);
                if ((int)r.out.size() >= r.max_new) retire(s, r);
            }
        }
        int active = (int)s->waiting.size();
        for (int b = 0; b < s->slots; ++b) active += s->slot_req[b] >= 0;
        *n_active = active;
    });
}

int at_sched_result(at_sched* s, int request_id, int* tokens_host, int cap, int* n_tokens, int* done) {
    return guard([&] {
        AT_REQUIRE(s && n_tokens && done && (cap == 0 || tokens_host), AT_ERR_INVALID_ARG, "null argument");
        auto it = s->reqs.find(request_id);
        AT_REQUIRE(it != s->reqs.end(), AT_ERR_INVALID_ARG, "unknown request id " + std::to_string(request_id));
        const Request& r = it->second;
        const int n = std::min<int>(cap, (int)r.out.size());
        for (int i = 0; i < n; ++i) tokens_host[i] = r.out[i];
        *n_tokens = (int)r.out.size();
        *done = r.done ? 1 : 0;
    });
}

}  // extern "C"
