// CPU ORACLE internals shared by ref_sampler.cpp and ref_mtp.cpp (test
// infrastructure only).
#ifndef TQF_REF_INTERNAL_H
#define TQF_REF_INTERNAL_H
#include <stdint.h>
#include <vector>
#include "ref_sampler.h"

namespace orc {
struct Cand {
    uint32_t token;
    float value;
};
// The full `sample` chain; kept_out receives the post-filter list in draw
// order (src/sampling/mod.rs:84-106 up to the draw).
uint32_t sample_core(const float* logits, int64_t n, const uint32_t* history,
                     int64_t hist_len, const orc_params* p, const float* u,
                     uint64_t* rng, std::vector<Cand>* kept_out, orc_debug* dbg);
}  // namespace orc
#endif
