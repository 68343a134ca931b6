// CPU ORACLE — test infrastructure only. Stochastic MTP verification over
// the sampler's post-filter distributions; see orc_mtp_verify in
// ref_sampler.h for the rule and the arithmetic it pins.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "ref_internal.h"
#include "ref_sampler.h"

namespace {

inline bool penalties_active(const orc_params* p) {
    return !(p->repeat_penalty == 1.0f && p->frequency_penalty == 0.0f &&
             p->presence_penalty == 0.0f);
}

// q as a dense vector: kept probabilities divided by the draw total (f32),
// or a point mass where the sampler's choice involves no uniform.
void filtered(const float* logits, int64_t n, const orc_params* p, std::vector<float>& q) {
    q.assign(static_cast<size_t>(n), 0.0f);
    if (n == 0) return;
    if (p->temperature == 0.0f) {
        uint32_t t[4];
        float v[4];
        orc_top_logit_candidates(logits, n, t, v);
        q[t[0]] = 1.0f;
        return;
    }
    std::vector<orc::Cand> kept;
    orc_debug dbg;
    std::memset(&dbg, 0, sizeof(dbg));
    const float u0 = 0.0f;
    orc::sample_core(logits, n, nullptr, 0, p, &u0, nullptr, &kept, &dbg);
    float total2 = -0.0f;
    for (const auto& c : kept) total2 += c.value;
    if (kept.empty()) { q[0] = 1.0f; return; }
    if (!std::isfinite(total2) || total2 <= 0.0f) { q[kept[0].token] = 1.0f; return; }
    for (const auto& c : kept) q[c.token] = c.value / total2;
}

// The residual draw: r_i = max(0, qt_i - qd_i) rounded to 2^-62 fixed point
// (round-half-even), summed exactly; thr = floor(floor(u*2^32) * R / 2^32);
// the first id (ascending) whose inclusive prefix exceeds thr.
int64_t residual_draw(const std::vector<float>& qt, const std::vector<float>& qd, float u) {
    const size_t n = qt.size();
    std::vector<uint64_t> r(n);
    unsigned __int128 total = 0;
    for (size_t i = 0; i < n; ++i) {
        const float d = qt[i] - qd[i];
        r[i] = d > 0.0f ? static_cast<uint64_t>(std::nearbyint(std::ldexp(static_cast<double>(d), 62)))
                        : 0ull;
        total += r[i];
    }
    if (total == 0) return -1;
    const uint64_t uq = static_cast<uint64_t>(std::ldexp(static_cast<double>(u), 32));
    const unsigned __int128 thr = (static_cast<unsigned __int128>(uq) * total) >> 32;
    unsigned __int128 pre = 0;
    for (size_t i = 0; i < n; ++i) {
        pre += r[i];
        if (pre > thr) return static_cast<int64_t>(i);
    }
    return static_cast<int64_t>(n) - 1;
}

}  // namespace

extern "C" {

void orc_filtered_distribution(const float* logits, int64_t n, const orc_params* params,
                               float* q_out) {
    std::vector<float> q;
    filtered(logits, n, params, q);
    std::copy(q.begin(), q.end(), q_out);
}

int orc_mtp_verify(const float* target, const float* draft, int64_t seqs, int64_t L,
                   int64_t n, int64_t ld, const uint32_t* drafts, const orc_params* params,
                   const float* uniforms, int32_t* out_accepted, int32_t* out_token,
                   uint8_t* out_mask, int threads) {
    for (int64_t s = 0; s < seqs; ++s)
        if (penalties_active(params + s)) return -1;
    if (threads <= 0) threads = static_cast<int>(std::thread::hardware_concurrency());
    threads = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(threads, seqs)));
    std::atomic<int64_t> next{0};
    auto worker = [&]() {
        std::vector<float> qt, qd;
        for (;;) {
            const int64_t s = next.fetch_add(1);
            if (s >= seqs) break;
            const orc_params* p = params + s;
            const float* us = uniforms + s * (L + 1);
            int32_t accepted = -1;
            int32_t token = 0;
            for (int64_t j = 0; j < L; ++j) {
                const float* trow = target + (s * (L + 1) + j) * ld;
                const float* drow = draft + (s * L + j) * ld;
                const uint32_t x = drafts[s * L + j];
                bool ok;
                if (p->temperature == 0.0f) {
                    // verify_pair (src/runtime/mtp.rs:98-104).
                    uint32_t t[4];
                    float v[4];
                    orc_top_logit_candidates(trow, n, t, v);
                    ok = orc_verify_pair(t[0], x) == 2;
                    if (!ok && accepted < 0) { accepted = static_cast<int32_t>(j); token = t[0]; }
                } else {
                    filtered(trow, n, p, qt);
                    filtered(drow, n, p, qd);
                    const float at = x < static_cast<uint64_t>(n) ? qt[x] : 0.0f;
                    const float ad = x < static_cast<uint64_t>(n) ? qd[x] : 0.0f;
                    ok = us[j] * ad < at;
                    if (!ok && accepted < 0) {
                        accepted = static_cast<int32_t>(j);
                        const int64_t t = residual_draw(qt, qd, us[L]);
                        if (t >= 0) {
                            token = static_cast<int32_t>(t);
                        } else {  // no residual mass: draw from the target itself
                            uint64_t dummy[4] = {0, 0, 0, 0};
                            token = static_cast<int32_t>(orc::sample_core(
                                trow, n, nullptr, 0, p, us + L, dummy, nullptr, nullptr));
                        }
                    }
                }
                if (out_mask) out_mask[s * L + j] = ok ? 1 : 0;
            }
            if (accepted < 0) {  // all drafts accepted: bonus draw from row L
                accepted = static_cast<int32_t>(L);
                const float* trow = target + (s * (L + 1) + L) * ld;
                if (p->temperature == 0.0f) {
                    uint32_t t[4];
                    float v[4];
                    orc_top_logit_candidates(trow, n, t, v);
                    token = static_cast<int32_t>(t[0]);
                } else {
                    uint64_t dummy[4] = {0, 0, 0, 0};
                    token = static_cast<int32_t>(orc::sample_core(trow, n, nullptr, 0, p,
                                                                  us + L, dummy, nullptr, nullptr));
                }
            }
            out_accepted[s] = accepted;
            out_token[s] = token;
        }
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < threads; ++t) pool.emplace_back(worker);
    worker();
    for (auto& th : pool) th.join();
    return 0;
}

}  // extern "C"
