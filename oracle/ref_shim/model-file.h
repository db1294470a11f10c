// Test infrastructure only: a stand-in for the reference's ModelFile so that its sampler sources
// (src/common/sampling.cpp, src/families/qwen3-tts/sampler.cpp, src/families/haru/sampler.cpp,
// src/families/drama3/sampler.cpp) compile
// without GGUF loading. The sampler functions this oracle calls (sample, candidates, pick, uniform,
// haru::candidates, drama3::candidates) never touch a ModelFile; only the Generation / file_* constructors do, and those
// throw here. Getter names and signatures follow src/common/model-file.h:90-114 of the reference.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

class ModelFile {
public:
    [[noreturn]] static void absent(const std::string & key) {
        throw std::logic_error("the sampler oracle has no model file (asked for " + key + ")");
    }
    uint32_t u32(const std::string & key) const { absent(key); }
    int size(const std::string & key) const { absent(key); }
    float f32(const std::string & key) const { absent(key); }
    double f64(const std::string & key) const { absent(key); }
    bool boolean(const std::string & key) const { absent(key); }
    std::vector<int32_t> i32_array(const std::string & key) const { absent(key); }
};
