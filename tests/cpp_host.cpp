// A C++17 host of libsttb200 through include/stt_b200.hpp, the mirror of the stt-wasm types.
// Uses only calls that need no device; each subcommand prints what the test compares:
//   cpp_host config                      the SttConfig defaults
//   cpp_host load <gguf>                 SttModel::from_shards with the default config: the Error's
//                                        status and text (the loader validates before any device use)
//   cpp_host q4bad                       Q4Tensor::from_q4_bytes with a wrong byte count: the Error
//   cpp_host spm <model> <id>...         SpmDecoder::load, vocab_len and decode
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iterator>

#include "stt_b200.hpp"

using namespace stt_web;

int main(int argc, char** argv) {
    const std::string cmd = argc > 1 ? argv[1] : "";
    try {
        if (cmd == "config") {
            const SttConfig c;
            std::printf("%d %d %d %d %d %d %d %d %d %d %.1f %d %d %u %u\n", c.num_layers, c.hidden_size, c.num_heads,
                        c.num_kv_heads, c.intermediate_size, c.vocab_size, c.text_in_vocab_size, c.num_codebooks,
                        c.audio_vocab_size, c.text_delay, c.rope_theta, c.max_seq_len, c.sliding_window,
                        c.text_padding_id, c.text_start_token);
            return 0;
        }
        if (cmd == "load" && argc == 3) {
            std::ifstream f(argv[2], std::ios::binary);
            std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
            // two shards, split in the middle (ShardedCursor, gguf.rs:321-397)
            const size_t half = bytes.size() / 2;
            std::vector<std::vector<uint8_t>> shards{{bytes.begin(), bytes.begin() + half}, {bytes.begin() + half, bytes.end()}};
            try {
                SttModel m = SttModel::from_shards(shards);
                std::printf("loaded\n");
            } catch (const Error& e) {
                std::printf("%d %s\n", e.code(), e.what());
            }
            return 0;
        }
        if (cmd == "q4bad") {
            try {
                Q4Tensor t = Q4Tensor::from_q4_bytes(std::vector<uint8_t>(18 * 4 - 1), 2, 64);
                std::printf("created\n");
            } catch (const Error& e) {
                std::printf("%d %s\n", e.code(), e.what());
            }
            return 0;
        }
        if (cmd == "spm" && argc >= 3) {
            const SpmDecoder d = SpmDecoder::load(argv[2]);
            std::vector<uint32_t> ids;
            for (int i = 3; i < argc; ++i) ids.push_back((uint32_t)std::strtoul(argv[i], nullptr, 10));
            std::printf("%zu\n%s\n", d.vocab_len(), d.decode(ids).c_str());
            return 0;
        }
    } catch (const Error& e) {
        std::fprintf(stderr, "%s\n", e.what());
        return 1;
    }
    std::fprintf(stderr, "usage: cpp_host config | load <gguf> | q4bad | spm <model> <id>...\n");
    return 2;
}
