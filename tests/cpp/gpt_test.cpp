// The reference's GPT parity test (src/main.cpp:19-66: compare(), gpt_test())
// written against the B200 library through the C++ adapter.  Reads a golden
// fixture bundle in the MIT2 container (tensor names as in the reference's
// fixture: prefix.<L>.tokens/.language/.embeddings, decode.prefill.logits,
// decode.<i>.code/.logits, generation.greedy.codes, generation.beam.codes) and
// prints one JSON line per case.  Exit code 0 when every case passes.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <iostream>
#include <string>
#include <vector>

#include "gpt_decoder.hpp"
#include "mit2_bundle.hpp"

static bool compare(const std::string& name, const std::vector<float>& actual, const std::vector<float>& expected,
                    float tolerance = 1e-4f, double rms_tolerance = 1e-5) {
    if (actual.size() != expected.size()) throw std::runtime_error("Output shape mismatch: " + name);
    double sum = 0, square = 0;
    float peak = 0;
    for (size_t i = 0; i < actual.size(); i++) {
        if (!std::isfinite(actual[i]) || !std::isfinite(expected[i])) throw std::runtime_error("Non-finite output: " + name);
        const float d = std::abs(actual[i] - expected[i]);
        peak = std::max(peak, d);
        sum += d;
        square += double(d) * d;
    }
    const double mean = sum / actual.size(), rmse = std::sqrt(square / actual.size());
    const bool pass = peak < tolerance && rmse < rms_tolerance;
    std::cout << "{\"case\":\"" << name << "\",\"max_abs_error\":" << peak << ",\"mean_abs_error\":" << mean
              << ",\"rmse\":" << rmse << ",\"pass\":" << (pass ? "true" : "false") << "}\n";
    return pass;
}

int main(int argc, char** argv) {
    if (argc != 3) {
        std::cerr << "usage: gpt_test MODEL_BUNDLE GOLDEN_BUNDLE\n";
        return 2;
    }
    try {
        itts::Mit2Bundle fixture(argv[2]);
        auto f32 = [&](const std::string& n) {
            const auto& t = fixture.info(n);
            std::vector<float> v(t.nbytes / 4);
            std::memcpy(v.data(), fixture.data(t), t.nbytes);
            return v;
        };
        auto u32 = [&](const std::string& n) {
            const auto& t = fixture.info(n);
            std::vector<uint32_t> v(t.nbytes / 4);
            std::memcpy(v.data(), fixture.data(t), t.nbytes);
            return v;
        };
        itts25b200::GptDecoder gpt(argv[1]);
        bool pass = true;
        std::vector<float> first;
        for (const char* lang : {"L3", "L41"}) {
            const std::string name = std::string("prefix.") + lang;
            auto prefix = gpt.prepare(f32("speaker"), f32("emotion"), u32(name + ".tokens"), u32(name + ".language")[0]);
            pass = compare(name, prefix, f32(name + ".embeddings")) && pass;
            if (first.empty()) first = std::move(prefix);
        }
        auto check_logits = [&](const std::string& name, const std::vector<float>& logits) {
            const auto ref = f32(name + ".logits");
            auto argmax = [](const std::vector<float>& x) { return std::max_element(x.begin(), x.end()) - x.begin(); };
            const bool match = argmax(logits) == argmax(ref);
            std::cout << "{\"case\":\"" << name << ".argmax\",\"exact_match\":" << (match ? "true" : "false") << "}\n";
            return compare(name, logits, ref, 1e-4f, 2e-5) && match;
        };
        pass = check_logits("decode.prefill", gpt.prefill(first)) && pass;
        for (uint32_t i = 1; i <= 4; i++) {
            const auto name = "decode." + std::to_string(i);
            pass = check_logits(name, gpt.step(u32(name + ".code")[0], i)) && pass;
        }
        itts25b200::GenerationOptions config;
        config.do_sample = false;
        config.repetition_penalty = 1;
        auto generated = gpt.generate(first, config, 8);
        const bool generated_match = generated.codes == u32("generation.greedy.codes");
        pass = generated_match && pass;
        std::cout << "{\"case\":\"generation.greedy\",\"exact_match\":" << (generated_match ? "true" : "false") << "}\n";
        config.num_beams = 3;
        auto beam = gpt.generate(first, config, 8);
        const bool beam_match = beam.codes == u32("generation.beam.codes");
        pass = beam_match && pass;
        std::cout << "{\"case\":\"generation.beam\",\"exact_match\":" << (beam_match ? "true" : "false") << "}\n";
        std::cout << "{\"stage\":\"gpt_2.5_b200\",\"cached_tokens\":" << gpt.cached_tokens()
                  << ",\"gpu_launches\":" << gpt.launch_count() << ",\"pass\":" << (pass ? "true" : "false") << "}\n";
        return pass && gpt.launch_count() > 0 ? 0 : 1;
    } catch (const std::exception& e) {
        std::cerr << "gpt_test: " << e.what() << '\n';
        return 1;
    }
}
