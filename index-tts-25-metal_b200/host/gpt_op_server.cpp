// The `gpt` operation of the reference's line-protocol server
// (src/server.cpp:16-56, op at :41-47) served by the B200 library.
//
//   itts_gpt_op_server <model bundle dir> [device]
//
// Prints {"ready":true,"backend":"b200","model":"2.5"}, then reads lines
// "op<TAB>input bundle<TAB>output file" from stdin.  For op `gpt` the input
// bundle (MIT2, no target check) holds config f32[8] = {do_sample,
// temperature, top_k, top_p, repetition_penalty, num_beams, length_penalty,
// max_tokens}, seed u32[2] (low, high word), speaker f32[192], emotion
// f32[1280], text u32[n] and language u32[1]; the op runs prepare and
// generate through the GptDecoder adapter, appends the stop code 8193 when the
// loop stopped, writes the codes as u32 to the output file and prints
// {"ok":true,"dtype":"u32","shape":[1,n],"gpu_launches":...,"seconds":...}.
// Failures print {"ok":false,"error":"..."} with the reference's messages.
// The other ops of the reference server belong to models this library does
// not hold and are answered with an error.
#include <chrono>
#include <cstdint>
#include <cstdlib>
#include <memory>
#include <fstream>
#include <iostream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "gpt_decoder.hpp"
#include "mit2_bundle.hpp"

namespace {

std::string json_string(const std::string& value) {
    std::string out = "\"";
    for (unsigned char c : value) {
        if (c == '"' || c == '\\') {
            out += '\\';
            out += char(c);
        } else if (c < 32) {
            out += ' ';
        } else {
            out += char(c);
        }
    }
    return out + '"';
}

std::vector<float> f32_tensor(const itts::Mit2Bundle& b, const std::string& name) {
    const auto& t = b.info(name);
    if (t.dtype != "f32") throw std::invalid_argument("Expected f32 tensor: " + name);
    const float* p = reinterpret_cast<const float*>(b.data(t));
    return std::vector<float>(p, p + t.nbytes / 4);
}

std::vector<uint32_t> u32_tensor(const itts::Mit2Bundle& b, const std::string& name) {
    const auto& t = b.info(name);
    if (t.dtype != "u32") throw std::invalid_argument("Expected u32 tensor: " + name);
    const uint32_t* p = reinterpret_cast<const uint32_t*>(b.data(t));
    return std::vector<uint32_t>(p, p + t.nbytes / 4);
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        std::cerr << "usage: " << argv[0] << " <model bundle dir> [device]" << std::endl;
        return 2;
    }
    std::unique_ptr<itts25b200::GptDecoder> gpt;
    try {
        gpt = std::make_unique<itts25b200::GptDecoder>(argv[1], argc > 2 ? std::atoi(argv[2]) : 0);
    } catch (const std::exception& e) {
        std::cout << "{\"ready\":false,\"error\":" << json_string(e.what()) << "}" << std::endl;
        return 1;
    }
    std::cout << "{\"ready\":true,\"backend\":\"b200\",\"model\":\"2.5\"}" << std::endl;
    std::string line;
    while (std::getline(std::cin, line)) {
        try {
            std::istringstream fields(line);
            std::string op, input_path, output_path, extra;
            if (!std::getline(fields, op, '\t') || !std::getline(fields, input_path, '\t') ||
                !std::getline(fields, output_path, '\t') || std::getline(fields, extra, '\t'))
                throw std::invalid_argument("Expected operation, input bundle and output file");
            const uint64_t before = gpt->launch_count();
            const auto start = std::chrono::steady_clock::now();
            std::vector<uint32_t> ids;
            if (op == "gpt") {
                itts::Mit2Bundle input(input_path);
                input.check_sizes();
                const auto config = f32_tensor(input, "config");
                const auto seed = u32_tensor(input, "seed");
                if (config.size() != 8 || seed.size() != 2) throw std::invalid_argument("Invalid generation config");
                itts25b200::GenerationOptions options;
                options.do_sample = config[0] != 0;
                options.temperature = config[1];
                options.top_k = static_cast<uint32_t>(config[2]);
                options.top_p = config[3];
                options.repetition_penalty = config[4];
                options.num_beams = static_cast<uint32_t>(config[5]);
                options.length_penalty = config[6];
                options.seed = uint64_t(seed[0]) | (uint64_t(seed[1]) << 32);
                const auto language = u32_tensor(input, "language");
                if (language.size() != 1) throw std::invalid_argument("Expected scalar: language");
                const auto prefix = gpt->prepare(f32_tensor(input, "speaker"), f32_tensor(input, "emotion"),
                                                 u32_tensor(input, "text"), language[0]);
                auto generated = gpt->generate(prefix, options, static_cast<uint32_t>(config[7]));
                ids = std::move(generated.codes);
                if (generated.stopped) ids.push_back(ITTS_GPT_STOP_CODE);
                if (ids.empty()) throw std::runtime_error("Empty generated speech");
            } else if (op == "qwen" || op == "speech" || op == "camp" || op == "emotion" || op == "codec" ||
                       op == "regulate" || op == "flow" || op == "vocode") {
                throw std::invalid_argument("Operation not served by the B200 GPT library: " + op);
            } else {
                throw std::invalid_argument("Unknown native operation: " + op);
            }
            std::ofstream out(output_path, std::ios::binary);
            if (!out) throw std::runtime_error("Cannot create operation output");
            out.write(reinterpret_cast<const char*>(ids.data()), std::streamsize(ids.size() * 4));
            out.close();
            if (!out) throw std::runtime_error("Native output write failed");
            std::cout << "{\"ok\":true,\"dtype\":\"u32\",\"shape\":[1," << ids.size()
                      << "],\"gpu_launches\":" << gpt->launch_count() - before << ",\"seconds\":"
                      << std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count() << "}"
                      << std::endl;
        } catch (const std::exception& e) {
            std::cout << "{\"ok\":false,\"error\":" << json_string(e.what()) << "}" << std::endl;
        }
    }
    return 0;
}
