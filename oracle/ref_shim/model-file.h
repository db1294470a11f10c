// Test infrastructure only: a stand-in for the reference's ModelFile so that its sampler sources
// (src/common/sampling.cpp, src/families/qwen3-tts/sampler.cpp, src/families/haru/sampler.cpp,
// src/families/drama3/sampler.cpp) compile without GGUF loading. The sampler functions the oracle calls
// (sample, candidates, pick, uniform, haru::candidates, drama3::candidates) never touch a ModelFile. A
// stub holds the scalar keys a test sets (set()), so that the reference's own Generation constructor
// (qwen3-tts/sampler.cpp:55-60) and Generation::banned can run; any other key throws. Getter names and
// signatures follow src/common/model-file.h:90-119 of the reference.
#pragma once

#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

class ModelFile {
public:
    [[noreturn]] static void absent(const std::string & key) {
        throw std::logic_error("the sampler oracle has no model file key " + key);
    }
    void set(const std::string & key, double value) { values_[key] = value; }
    uint32_t u32(const std::string & key) const { return (uint32_t) get(key); }
    int size(const std::string & key) const { return (int) get(key); }
    float f32(const std::string & key) const { return (float) get(key); }
    double f64(const std::string & key) const { return get(key); }
    bool boolean(const std::string & key) const { return get(key) != 0.0; }
    std::vector<int32_t> i32_array(const std::string & key) const { absent(key); }

private:
    double get(const std::string & key) const {
        const auto it = values_.find(key);
        if (it == values_.end()) absent(key);
        return it->second;
    }
    std::map<std::string, double> values_;
};
