// Test infrastructure only: a CPU restatement of the reference's top-k sampling step
// (topk_sample, src/gten/sampler.cpp:63-128) with the generator seeded by the caller instead of
// std::random_device (sampler.cpp:70-71), so that draws are reproducible. It uses the same standard
// library pieces as the reference (std::partial_sort, std::exp, std::discrete_distribution,
// std::mt19937 of libstdc++), which is what makes it the checker of the device sampler.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <random>
#include <utility>
#include <vector>

namespace {

// One step of topk_sample (sampler.cpp:90-128) on n logits with generator gen; temp and top_k
// already clamped as sampler.cpp:66-67.
int topk_step(const float* row, int n, float temp, int top_k, std::mt19937& gen) {
    std::vector<std::pair<double, int>> cand;
    cand.reserve(n);
    for (int j = 0; j < n; ++j) cand.push_back(std::make_pair((double)row[j] / temp, j));
    std::partial_sort(cand.begin(), cand.begin() + top_k, cand.end(),
                      [](const std::pair<double, int>& a, const std::pair<double, int>& b) {
                          return a.first > b.first;  // descending, the reference's comparator
                      });
    cand.resize(top_k);
    double z = 0;
    for (int j = 0; j < top_k; ++j) {
        cand[j].first = std::exp(cand[j].first);
        z += cand[j].first;
    }
    for (int j = 0; j < top_k; ++j) cand[j].first = cand[j].first / z;
    std::vector<double> weight(n, 0.0);  // the vocabulary-sized probability vector
    for (const auto& c : cand) weight[c.second] = c.first;
    std::discrete_distribution<int> pick(weight.begin(), weight.end());
    return pick(gen);
}

bool clamp_args(int n, float& temp, int& top_k) {
    top_k = std::min(top_k, 1000);
    temp = std::min(temp, 2.0f);
    return n >= 1 && top_k >= 1 && top_k <= n && temp > 0.0f;
}

}  // namespace

extern "C" {

// Runs n_draws steps with one generator std::mt19937(seed); step d samples from the n logits at
// logits + d * n. temp and top_k are clamped as sampler.cpp:66-67. Returns 0, or -1 on bad input.
int or_topk_sample(const float* logits, int n, float temp, int top_k, uint32_t seed, int n_draws, int32_t* out) {
    if (!clamp_args(n, temp, top_k)) return -1;
    std::mt19937 gen(seed);
    for (int d = 0; d < n_draws; ++d) out[d] = topk_step(logits + (long)d * n, n, temp, top_k, gen);
    return 0;
}

// A generator that persists across steps, for decode loops whose next logits depend on the draw:
// or_sampler_new(seed), then or_sampler_step per step (returns the id, or -1 on bad input).
void* or_sampler_new(uint32_t seed) { return new std::mt19937(seed); }

int or_sampler_step(void* h, const float* logits, int n, float temp, int top_k) {
    if (!clamp_args(n, temp, top_k)) return -1;
    return topk_step(logits, n, temp, top_k, *static_cast<std::mt19937*>(h));
}

void or_sampler_free(void* h) { delete static_cast<std::mt19937*>(h); }

}  // extern "C"

extern "C" {

// The first n outputs of std::mt19937(seed) (checks the generator restated on the device).
void or_mt19937(uint32_t seed, int n, uint32_t* out) {
    std::mt19937 gen(seed);
    for (int i = 0; i < n; ++i) out[i] = gen();
}

}  // extern "C"
