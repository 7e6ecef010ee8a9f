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

extern "C" {

// Runs n_draws steps with one generator std::mt19937(seed); step d samples from the n logits at
// logits + d * n. temp and top_k are clamped as sampler.cpp:66-67. Returns 0, or -1 on bad input.
int or_topk_sample(const float* logits, int n, float temp, int top_k, uint32_t seed, int n_draws, int32_t* out) {
    top_k = std::min(top_k, 1000);
    temp = std::min(temp, 2.0f);
    if (n < 1 || top_k < 1 || top_k > n || !(temp > 0.0f)) return -1;
    std::mt19937 gen(seed);
    std::vector<std::pair<double, int>> cand;
    for (int d = 0; d < n_draws; ++d) {
        const float* row = logits + (long)d * n;
        cand.clear();
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
        out[d] = pick(gen);
    }
    return 0;
}

}  // extern "C"

extern "C" {

// The first n outputs of std::mt19937(seed) (checks the generator restated on the device).
void or_mt19937(uint32_t seed, int n, uint32_t* out) {
    std::mt19937 gen(seed);
    for (int i = 0; i < n; ++i) out[i] = gen();
}

}  // extern "C"
