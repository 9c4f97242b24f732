// rocket_h_check.cpp -- test driver: calls the rocket.h C++ API (reference
// rocket.h:36-50) of librkv_b200.so on plain host buffers, as a C++ caller of
// the reference library does, and writes the results for tests/test_gpu_dropin.py.
//
//   rocket_h_check evict  DIR  args.txt "H HK D window kernel budget len_q len_k",
//                              Q.f32, K.f32           -> kept.i32
//   rocket_h_check decode DIR  args.txt "H HK D topk chunk r cr len_k",
//                              Q.f32, K.f32, V.f32    -> O.f32
//   rocket_h_check params DIR  args.txt "budget seq max_new head_dim window"
//                                                     -> params.txt (9 numbers)
//   rocket_h_check bad    DIR  a config the reference cannot size
//                                                     -> prints the exception type
// Exit status 0 on success, 2 when a rocket.h call threw (message on stderr).
#include <cstdio>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "rocket.h"

namespace {

std::vector<char> read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot read " + path);
    return std::vector<char>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

template <typename T>
std::vector<T> read_array(const std::string& path) {
    const std::vector<char> b = read_file(path);
    std::vector<T> v(b.size() / sizeof(T));
    std::copy(b.begin(), b.begin() + v.size() * sizeof(T), reinterpret_cast<char*>(v.data()));
    return v;
}

template <typename T>
void write_array(const std::string& path, const std::vector<T>& v) {
    std::ofstream f(path, std::ios::binary);
    f.write(reinterpret_cast<const char*>(v.data()), (std::streamsize)(v.size() * sizeof(T)));
    if (!f) throw std::runtime_error("cannot write " + path);
}

std::ifstream args_of(const std::string& dir) {
    std::ifstream a(dir + "/args.txt");
    if (!a) throw std::runtime_error("cannot read " + dir + "/args.txt");
    return a;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc != 3) {
        std::fprintf(stderr, "usage: %s evict|decode|params|bad DIR\n", argv[0]);
        return 1;
    }
    const std::string mode = argv[1], dir = argv[2];
    try {
        if (mode == "evict") {
            RocketConfig cfg{};
            int len_q = 0, len_k = 0;
            args_of(dir) >> cfg.num_heads >> cfg.num_heads_kv >> cfg.dim_head >> cfg.window_size >>
                cfg.kernel_size >> cfg.prompt_budget >> len_q >> len_k;
            const std::vector<float> Q = read_array<float>(dir + "/Q.f32"), K = read_array<float>(dir + "/K.f32");
            const std::vector<int> kept = compute_prefill_eviction(Q.data(), K.data(), len_q, len_k, cfg);
            write_array(dir + "/kept.i32", kept);
        } else if (mode == "decode") {
            RocketConfig cfg{};
            int len_k = 0;
            args_of(dir) >> cfg.num_heads >> cfg.num_heads_kv >> cfg.dim_head >> cfg.topk_decode >> cfg.chunk_size >>
                cfg.r_dim >> cfg.compression_ratio >> len_k;
            const std::vector<float> Q = read_array<float>(dir + "/Q.f32"), K = read_array<float>(dir + "/K.f32"),
                                     V = read_array<float>(dir + "/V.f32");
            write_array(dir + "/O.f32", compute_hybrid_sparse_decode(Q.data(), K.data(), V.data(), len_k, cfg));
        } else if (mode == "params") {
            int budget = 0, seq = 0, max_new = 0, head_dim = 0, window = 0;
            args_of(dir) >> budget >> seq >> max_new >> head_dim >> window;
            const RocketBudgetParams p = compute_rocket_params(budget, seq, max_new, head_dim, window);
            std::ofstream o(dir + "/params.txt");
            o << p.token_budget << ' ' << p.sequence_length << ' ' << p.max_new_tokens << ' ' << p.capacity_budget
              << ' ' << p.prompt_budget << ' ' << p.chunk_size << ' ' << p.r << ' ' << p.k << ' ';
            o.precision(9);
            o << p.compression_ratio << '\n';
        } else if (mode == "bad") {
            RocketConfig cfg{};  // num_heads_kv 0: the reference cannot form its groups
            cfg.num_heads = 24;
            cfg.dim_head = 128;
            cfg.prompt_budget = 16;
            std::vector<float> Q(24 * 64 * 128), K(64 * 128);
            try {
                compute_prefill_eviction(Q.data(), K.data(), 64, 64, cfg);
                std::printf("no exception\n");
            } catch (const std::invalid_argument&) {
                std::printf("invalid_argument\n");
            } catch (const std::runtime_error&) {
                std::printf("runtime_error\n");
            }
        } else {
            std::fprintf(stderr, "unknown mode %s\n", mode.c_str());
            return 1;
        }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "rocket.h call failed: %s\n", e.what());
        return 2;
    }
    return 0;
}
