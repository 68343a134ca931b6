// CPU ORACLE — test infrastructure only (see ref_sampler.h for scope, pins
// and the reference lines each function restates). Compiled with
// -O3 -ffp-contract=off so every f32 operation rounds exactly as the Rust
// reference's separate operations do; expf is glibc's, as Rust's f32::exp
// uses on Linux.
#include "ref_sampler.h"
#include "ref_internal.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <limits>
#include <thread>
#include <unordered_map>
#include <vector>

namespace orc {

// compare_desc (src/sampling/mod.rs:258-266): -1 Less, 0 Equal, 1 Greater.
inline int compare_desc(float a, float b) {
    const bool an = std::isnan(a), bn = std::isnan(b);
    if (an && bn) return 0;
    if (an) return 1;   // a is NaN: sorts after b
    if (bn) return -1;
    if (b < a) return -1;  // b.partial_cmp(&a)
    if (b > a) return 1;
    return 0;
}

// Total order (value desc NaN last, token asc): the sort key of
// src/sampling/mod.rs:188 and the pinned top-k tie policy.
inline bool before(const Cand& a, const Cand& b) {
    const int c = compare_desc(a.value, b.value);
    if (c != 0) return c < 0;
    return a.token < b.token;
}

inline float bf16_to_f32(uint16_t h) {
    const uint32_t bits = static_cast<uint32_t>(h) << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

// apply_penalties (src/sampling/mod.rs:114-148) over candidates in id order.
void penalise(std::vector<Cand>& cands, const uint32_t* history, int64_t hist_len,
              const orc_params* p) {
    const float repeat = p->repeat_penalty;
    const float frequency = p->frequency_penalty;
    const float presence = p->presence_penalty;
    if (repeat == 1.0f && frequency == 0.0f && presence == 0.0f) return;
    const uint64_t len = hist_len > 0 ? static_cast<uint64_t>(hist_len) : 0;
    const uint64_t window = std::min<uint64_t>(p->repeat_last_n, len);
    if (window == 0) return;
    const uint32_t* recent = history + (len - window);
    std::unordered_map<uint32_t, uint32_t> counts;
    counts.reserve(static_cast<size_t>(window) * 2);
    for (uint64_t i = 0; i < window; ++i) counts[recent[i]] += 1;
    for (Cand& c : cands) {
        auto it = counts.find(c.token);
        if (it == counts.end()) continue;
        if (repeat != 1.0f) c.value = (c.value > 0.0f) ? c.value / repeat : c.value * repeat;
        float t = frequency * static_cast<float>(it->second);
        t = t + presence;
        c.value = c.value - t;
    }
}

uint32_t sample_core(const float* logits, int64_t n, const uint32_t* history,
                     int64_t hist_len, const orc_params* p, const float* u,
                     uint64_t* rng, std::vector<Cand>* kept_out, orc_debug* dbg) {
    if (dbg) {
        dbg->n_after_topk = dbg->n_after_topp = dbg->n_after_minp = 0;
        dbg->total = dbg->total2 = dbg->target = 0.0f;
        dbg->consumed = 0;
        dbg->topk_tie = 0;
        dbg->drawn_index = -1;
        dbg->cdf_margin = dbg->topp_margin = std::numeric_limits<double>::infinity();
    }
    // sample (src/sampling/mod.rs:90-97): candidates in token order.
    std::vector<Cand> cands(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; ++i) cands[i] = Cand{static_cast<uint32_t>(i), logits[i]};
    penalise(cands, history, hist_len, p);

    // apply_top_k (src/sampling/mod.rs:153-161), ties resolved to low ids.
    const uint64_t k = p->top_k;
    if (k != 0 && k < static_cast<uint64_t>(cands.size())) {
        std::nth_element(cands.begin(), cands.begin() + (k - 1), cands.end(), before);
        if (dbg) {
            const float kth = cands[k - 1].value;
            for (size_t j = k; j < cands.size(); ++j)
                if (compare_desc(cands[j].value, kth) == 0) { dbg->topk_tie = 1; break; }
        }
        cands.resize(k);
        std::sort(cands.begin(), cands.end(), before);  // pinned summation order
    }
    if (dbg) dbg->n_after_topk = static_cast<int64_t>(cands.size());

    // softmax (src/sampling/mod.rs:166-190).
    float max = -std::numeric_limits<float>::infinity();
    for (const Cand& c : cands)
        if (c.value > max) max = c.value;  // f32::max ignores NaN
    std::vector<Cand> probs(cands.size());
    for (size_t i = 0; i < cands.size(); ++i) {
        const float x = (cands[i].value - max) / p->temperature;
        probs[i] = Cand{cands[i].token, expf(x)};
    }
    float total = -0.0f;  // Rust's `Sum for f32` folds from -0.0
    for (const Cand& c : probs) total += c.value;
    if (total > 0.0f)
        for (Cand& c : probs) c.value /= total;
    std::sort(probs.begin(), probs.end(), before);
    if (dbg) dbg->total = total;

    // apply_top_p (src/sampling/mod.rs:195-209).
    if (!(p->top_p >= 1.0f)) {
        float cumulative = 0.0f;
        float prev = 0.0f;
        size_t keep = 0;
        for (const Cand& c : probs) {
            prev = cumulative;
            cumulative += c.value;
            keep += 1;
            if (cumulative >= p->top_p) break;
        }
        if (dbg && keep > 0) {
            const double hi = static_cast<double>(cumulative) - p->top_p;
            const double lo = keep > 1 ? static_cast<double>(p->top_p) - prev
                                       : std::numeric_limits<double>::infinity();
            dbg->topp_margin = std::min(std::fabs(hi), std::fabs(lo));
        }
        keep = std::max<size_t>(keep, 1);
        if (keep < probs.size()) probs.resize(keep);
    }
    if (dbg) dbg->n_after_topp = static_cast<int64_t>(probs.size());

    // apply_min_p (src/sampling/mod.rs:213-224).
    if ((p->flags & 1u) && !(p->min_p <= 0.0f) && !probs.empty()) {
        const float floor = p->min_p * probs[0].value;
        size_t keep = 0;
        while (keep < probs.size() && probs[keep].value >= floor) ++keep;
        keep = std::max<size_t>(keep, 1);
        if (keep < probs.size()) probs.resize(keep);
    }
    if (dbg) dbg->n_after_minp = static_cast<int64_t>(probs.size());
    if (kept_out) *kept_out = probs;

    // draw (src/sampling/mod.rs:227-248).
    if (probs.empty()) return 0;
    float total2 = -0.0f;
    for (const Cand& c : probs) total2 += c.value;
    if (dbg) dbg->total2 = total2;
    if (!std::isfinite(total2) || total2 <= 0.0f) {
        if (dbg) dbg->drawn_index = 0;
        return probs[0].token;
    }
    const float uu = u ? *u : orc_xoshiro_next_f32(rng);
    if (dbg) dbg->consumed = 1;
    const float target = uu * total2;
    if (dbg) dbg->target = target;
    float cumulative = 0.0f;
    for (size_t i = 0; i < probs.size(); ++i) {
        const float before_cum = cumulative;
        cumulative += probs[i].value;
        if (cumulative >= target) {
            if (dbg) {
                dbg->drawn_index = static_cast<int64_t>(i);
                const double a = static_cast<double>(cumulative) - target;
                const double b = static_cast<double>(target) - before_cum;
                dbg->cdf_margin = std::min(a, i > 0 ? b : a) / total2;
            }
            return probs[i].token;
        }
    }
    if (dbg) dbg->drawn_index = static_cast<int64_t>(probs.size()) - 1;
    return probs.back().token;
}

}  // namespace orc

using orc::Cand;
using orc::sample_core;
using orc::bf16_to_f32;
using orc::rotl;

extern "C" {

// Xoshiro256PlusPlus::from_seed (src/sampling/mod.rs:283-295).
void orc_xoshiro_from_seed(uint64_t seed, uint64_t state[4]) {
    uint64_t z = seed;
    for (int i = 0; i < 4; ++i) {
        z += 0x9E3779B97F4A7C15ull;
        uint64_t x = z;
        x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
        x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
        state[i] = x ^ (x >> 31);
    }
}

// next_u64 (src/sampling/mod.rs:311-324).
uint64_t orc_xoshiro_next_u64(uint64_t s[4]) {
    const uint64_t result = rotl(s[0] + s[3], 23) + s[0];
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return result;
}

// next_f32 (src/sampling/mod.rs:328-330).
float orc_xoshiro_next_f32(uint64_t s[4]) {
    return static_cast<float>(orc_xoshiro_next_u64(s) >> 40) / static_cast<float>(1u << 24);
}

// top_logit_candidates (src/runtime/decode.rs:48-64).
void orc_top_logit_candidates(const float* logits, int64_t n, uint32_t tokens[4],
                              float values[4]) {
    for (int i = 0; i < 4; ++i) {
        tokens[i] = 0;
        values[i] = -std::numeric_limits<float>::infinity();
    }
    for (int64_t idx = 0; idx < n; ++idx) {
        const float v = logits[idx];
        int pos = -1;
        for (int i = 0; i < 4; ++i)
            if (v > values[i]) { pos = i; break; }
        if (pos < 0) continue;
        for (int i = 3; i > pos; --i) {
            tokens[i] = tokens[i - 1];
            values[i] = values[i - 1];
        }
        tokens[pos] = static_cast<uint32_t>(idx);
        values[pos] = v;
    }
}

void orc_apply_penalties(float* values, int64_t n, const uint32_t* history,
                         int64_t hist_len, const orc_params* params) {
    std::vector<Cand> cands(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; ++i) cands[i] = Cand{static_cast<uint32_t>(i), values[i]};
    penalise(cands, history, hist_len, params);
    for (int64_t i = 0; i < n; ++i) values[i] = cands[i].value;
}

uint32_t orc_sample(const float* logits, int64_t n, const uint32_t* history,
                    int64_t hist_len, const orc_params* params, const float* u,
                    uint64_t rng_state[4], orc_debug* dbg) {
    std::vector<Cand> kept;
    const bool want = dbg && dbg->kept_tokens && dbg->kept_probs;
    const uint32_t tok = sample_core(logits, n, history, hist_len, params, u, rng_state,
                                     want ? &kept : nullptr, dbg);
    if (want) {
        const int64_t m = std::min<int64_t>(dbg->kept_cap, static_cast<int64_t>(kept.size()));
        for (int64_t i = 0; i < m; ++i) {
            dbg->kept_tokens[i] = kept[i].token;
            dbg->kept_probs[i] = kept[i].value;
        }
    }
    return tok;
}

uint32_t orc_sample_dense(const float* logits, int64_t n, const uint32_t* history,
                          int64_t hist_len, const orc_params* params, const float* u,
                          uint64_t rng_state[4], float* probs_out, orc_debug* dbg) {
    std::vector<Cand> kept;
    const uint32_t tok =
        sample_core(logits, n, history, hist_len, params, u, rng_state, &kept, dbg);
    if (probs_out) {
        std::fill(probs_out, probs_out + n, 0.0f);
        for (const Cand& c : kept) probs_out[c.token] = c.value;
    }
    return tok;
}

void orc_sample_batch(const void* logits, int dtype, int64_t rows, int64_t n, int64_t ld,
                      const int32_t* hist, const int64_t* hist_off,
                      const orc_params* params, const float* uniforms,
                      uint64_t* rng_states, int32_t* out_tokens, int threads) {
    if (threads <= 0) threads = static_cast<int>(std::thread::hardware_concurrency());
    if (threads < 1) threads = 1;
    if (threads > rows) threads = static_cast<int>(std::max<int64_t>(rows, 1));
    std::atomic<int64_t> next{0};
    auto worker = [&]() {
        std::vector<float> row;
        if (dtype != 0) row.resize(static_cast<size_t>(n));
        for (;;) {
            const int64_t r = next.fetch_add(1);
            if (r >= rows) break;
            const float* lr;
            if (dtype == 0) {
                lr = static_cast<const float*>(logits) + r * ld;
            } else {
                const uint16_t* src = static_cast<const uint16_t*>(logits) + r * ld;
                for (int64_t i = 0; i < n; ++i) row[i] = bf16_to_f32(src[i]);
                lr = row.data();
            }
            const orc_params* p = params + r;
            if (p->temperature == 0.0f) {  // Sampler::new greedy arm
                uint32_t t[4];
                float v[4];
                orc_top_logit_candidates(lr, n, t, v);
                out_tokens[r] = static_cast<int32_t>(t[0]);
                continue;
            }
            const uint32_t* h = nullptr;
            int64_t hl = 0;
            if (hist && hist_off) {
                h = reinterpret_cast<const uint32_t*>(hist) + hist_off[r];
                hl = hist_off[r + 1] - hist_off[r];
            }
            out_tokens[r] = static_cast<int32_t>(
                sample_core(lr, n, h, hl, p, uniforms ? uniforms + r : nullptr,
                            rng_states ? rng_states + 4 * r : nullptr, nullptr, nullptr));
        }
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < threads; ++t) pool.emplace_back(worker);
    worker();
    for (auto& th : pool) th.join();
}

// verify_pair (src/runtime/mtp.rs:98-104).
int orc_verify_pair(uint32_t target_prediction, uint32_t draft_token) {
    return target_prediction == draft_token ? 2 : 1;
}

}  // extern "C"
