// Continuous-batching scheduler over one libqwen_b200 handle. The reference
// serves one request at a time (src/software/main.c:243-265: reset the
// context, qgen_run to completion, next prompt). Here requests queue up and
// share the GPU: every step
//   1. admits waiting requests into free sequence slots (FIFO);
//   2. feeds prompt tokens of admitted requests through one batched prefill
//      (qwen_b200_prefill), at most `prefill_budget` tokens per step, so a
//      long prompt is split over several steps (chunked prefill) and cannot
//      stall the running requests; a request whose prompt is complete gets
//      its first token from that prefill;
//   3. runs one batched decode step (qwen_b200_decode_step) for every
//      request that has a token and is not finished;
//   4. retires requests that reached max_new tokens or produced an
//      end-of-text id (151643 or 151645, the stop ids of
//      src/software/generation.c), freeing their slots.
// Each request's tokens are exactly those of the request run alone: slots are
// independent and every kernel's result is independent of the batch.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <deque>
#include <map>
#include <new>
#include <vector>

#include "qwen_b200.h"

namespace {

constexpr uint32_t kEos0 = 151643, kEos1 = 151645;

struct Request {
    uint32_t id = 0;
    std::vector<uint32_t> prompt;
    uint32_t fed = 0;  // prompt tokens already prefilled
    uint32_t max_new = 0;
    int slot = -1;
    std::vector<uint32_t> out;
    bool done = false;
};

}  // namespace

struct qwen_b200_sched {
    qwen_b200 *h = nullptr;
    uint32_t slots = 0, capacity = 0, budget = 0;
    uint32_t next_id = 1;
    std::map<uint32_t, Request> reqs;   // every request not yet collected
    std::deque<uint32_t> waiting;       // submitted, no slot yet
    std::vector<uint32_t> slot_owner;   // request id per slot, 0 = free
};

extern "C" {

int qwen_b200_sched_open(qwen_b200 *h, uint32_t prefill_budget, qwen_b200_sched **out) {
    if (!h || !out || prefill_budget == 0) return QWEN_B200_EINVAL;
    *out = nullptr;
    qwen_b200_config cfg;
    if (qwen_b200_get_config(h, &cfg)) return QWEN_B200_EINVAL;
    qwen_b200_sched *s = new (std::nothrow) qwen_b200_sched();
    if (!s) return QWEN_B200_ENOMEM;
    s->h = h;
    s->slots = cfg.max_seqs;
    s->capacity = cfg.max_context;
    const uint32_t n = cfg.max_seqs;
    s->budget = prefill_budget;
    s->slot_owner.assign(n, 0);
    *out = s;
    return QWEN_B200_OK;
}

int qwen_b200_sched_close(qwen_b200_sched *s) {
    if (!s) return QWEN_B200_EINVAL;
    delete s;
    return QWEN_B200_OK;
}

int qwen_b200_sched_submit(qwen_b200_sched *s, const uint32_t *ids, uint32_t n, uint32_t max_new,
                           uint32_t *request_id) {
    if (!s || !ids || n == 0 || max_new == 0 || !request_id) return QWEN_B200_EINVAL;
    for (uint32_t i = 0; i < n; ++i)
        if (ids[i] >= QWEN_B200_VOCAB) return QWEN_B200_EINVAL;
    if ((uint64_t)n + max_new > s->capacity) return QWEN_B200_ESTATE;  // would overflow a slot's KV cache
    Request r;
    r.id = s->next_id++;
    r.prompt.assign(ids, ids + n);
    r.max_new = max_new;
    const uint32_t id = r.id;
    s->reqs.emplace(id, std::move(r));
    s->waiting.push_back(id);
    *request_id = id;
    return QWEN_B200_OK;
}

int qwen_b200_sched_step(qwen_b200_sched *s, uint32_t *running) {
    if (!s) return QWEN_B200_EINVAL;
    qwen_b200 *h = s->h;
    // 1. admission
    for (uint32_t slot = 0; slot < s->slots && !s->waiting.empty(); ++slot) {
        if (s->slot_owner[slot]) continue;
        const uint32_t id = s->waiting.front();
        s->waiting.pop_front();
        Request &r = s->reqs[id];
        const int rc = qwen_b200_reset(h, slot);
        if (rc) return rc;
        r.slot = (int)slot;
        s->slot_owner[slot] = id;
    }
    // 2. chunked prefill of admitted prompts, within the token budget
    std::vector<uint32_t> pslots, plens, pids, pfinal;
    uint32_t used = 0;
    for (uint32_t slot = 0; slot < s->slots && used < s->budget; ++slot) {
        const uint32_t id = s->slot_owner[slot];
        if (!id) continue;
        Request &r = s->reqs[id];
        if (r.fed == r.prompt.size()) continue;
        const uint32_t take = std::min<uint32_t>((uint32_t)r.prompt.size() - r.fed, s->budget - used);
        pslots.push_back(slot);
        plens.push_back(take);
        pids.insert(pids.end(), r.prompt.begin() + r.fed, r.prompt.begin() + r.fed + take);
        pfinal.push_back(id);
        used += take;
    }
    if (!pslots.empty()) {
        std::vector<uint32_t> toks(pslots.size());
        const int rc = qwen_b200_prefill(h, (uint32_t)pslots.size(), pslots.data(), plens.data(), pids.data(),
                                         toks.data(), nullptr);
        if (rc) return rc;
        for (size_t i = 0; i < pslots.size(); ++i) {
            Request &r = s->reqs[pfinal[i]];
            r.fed += plens[i];
            if (r.fed == r.prompt.size()) r.out.push_back(toks[i]);  // the first generated token
        }
    }
    // 3. one decode step for every request that has a token and room for more
    std::vector<uint32_t> dslots, dtoks, downer;
    for (uint32_t slot = 0; slot < s->slots; ++slot) {
        const uint32_t id = s->slot_owner[slot];
        if (!id) continue;
        Request &r = s->reqs[id];
        if (r.out.empty() || r.done) continue;
        const uint32_t last = r.out.back();
        if (r.out.size() >= r.max_new || last == kEos0 || last == kEos1) continue;
        dslots.push_back(slot);
        dtoks.push_back(last);
        downer.push_back(id);
    }
    if (!dslots.empty()) {
        std::vector<uint32_t> out(dslots.size());
        const int rc = qwen_b200_decode_step(h, dslots.data(), dtoks.data(), (uint32_t)dslots.size(), out.data());
        if (rc) return rc;
        for (size_t i = 0; i < dslots.size(); ++i) s->reqs[downer[i]].out.push_back(out[i]);
    }
    // 4. retire finished requests
    uint32_t live = 0;
    for (uint32_t slot = 0; slot < s->slots; ++slot) {
        const uint32_t id = s->slot_owner[slot];
        if (!id) continue;
        Request &r = s->reqs[id];
        if (!r.out.empty() &&
            (r.out.size() >= r.max_new || r.out.back() == kEos0 || r.out.back() == kEos1)) {
            r.done = true;
            r.slot = -1;
            s->slot_owner[slot] = 0;
        } else {
            ++live;
        }
    }
    if (running) *running = live + (uint32_t)s->waiting.size();
    return QWEN_B200_OK;
}

int qwen_b200_sched_result(qwen_b200_sched *s, uint32_t request_id, uint32_t *tokens, uint32_t cap,
                           uint32_t *count, int *done) {
    if (!s || !count || !done) return QWEN_B200_EINVAL;
    auto it = s->reqs.find(request_id);
    if (it == s->reqs.end()) return QWEN_B200_EINVAL;
    const Request &r = it->second;
    *count = (uint32_t)r.out.size();
    *done = r.done ? 1 : 0;
    if (tokens) std::memcpy(tokens, r.out.data(), sizeof(uint32_t) * std::min<size_t>(cap, r.out.size()));
    if (r.done) s->reqs.erase(it);  // collected
    return QWEN_B200_OK;
}

}  // extern "C"
