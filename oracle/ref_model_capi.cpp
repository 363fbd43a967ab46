// TEST INFRASTRUCTURE ONLY: C entry points over the reference's own CPU Transformer
// (src/model.cpp, compiled from the reference sources by `make -C oracle ref`), the parity
// oracle for the tensor-parallel transformer: load a llama2.c checkpoint
// (load_checkpoint, model.cpp:113-169), run forward / prefill (model.cpp:247-322), and the
// RoPE tables (rope_tables, model.cpp:171-184) for pinning the library's own.
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

#include "model.h"

namespace {
thread_local std::string g_err;
}

extern "C" {

const char* ref_model_error() { return g_err.c_str(); }

// Returns an opaque handle, or NULL (message in ref_model_error()).
void* ref_model_load(const char* path, int q8) {
    try {
        Checkpoint ck = load_checkpoint(path);
        return new Transformer(std::move(ck), q8 ? WeightType::q8 : WeightType::f32);
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void ref_model_free(void* h) { delete static_cast<Transformer*>(h); }

size_t ref_model_vocab(void* h) { return static_cast<Transformer*>(h)->config().vocab_size; }

// Feeds tokens[0:n] at positions [pos, pos + n) (n == 1: forward, else prefill) and writes
// the logits of the last row into out (vocab floats). Returns 0, or 1 on error.
int ref_model_run(void* h, const int* tokens, size_t n, size_t pos, float* out) {
    try {
        auto* t = static_cast<Transformer*>(h);
        const std::vector<float>& l =
            n == 1 ? t->forward(tokens[0], pos) : t->prefill(std::vector<int>(tokens, tokens + n), pos);
        std::memcpy(out, l.data(), l.size() * sizeof(float));
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 1;
    }
}

void ref_rope_tables(size_t seq_len, size_t dim, size_t n_heads, float* cos, float* sin) {
    Config c{dim, 1, 1, n_heads, n_heads, 1, seq_len};
    std::vector<float> cv, sv;
    rope_tables(c, cv, sv);
    std::memcpy(cos, cv.data(), cv.size() * sizeof(float));
    std::memcpy(sin, sv.data(), sv.size() * sizeof(float));
}

}  // extern "C"
