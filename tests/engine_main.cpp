// Test driver for fpga_qwen_b200/host/qwen_forward.hpp (built and run by tests/test_engine.py):
// the reference engine's forward pass on the GPU through libqattn, over a synthetic checkpoint.
//   engine_main <weights.bin> <ids.bin> <logits.bin>
// weights.bin: int32 layers, hidden, intermediate, vocab; FP16 embedding [vocab][hidden];
// FP32 final norm [hidden]; per layer FP32 input norm [hidden], post-attention norm [hidden],
// q_norm [128], k_norm [128], then FP16 q [2048][hidden], k [1024][hidden], v [1024][hidden],
// o [hidden][2048], gate [inter][hidden], up [inter][hidden], down [hidden][inter].
// ids.bin: int32 token ids (13). The scenario: prefill ids[0..8), step ids[8], step ids[9],
// verify_two(ids[10], ids[11]) + commit_verified(2), step ids[12], truncate(5), prefill
// ids[5..9), step ids[9]. logits.bin: FP32 [8][vocab], the logits after each of those rows
// in order (a verification gives two rows). Prints the final position.
//   engine_main <weights.bin> <ids.bin> <logits.bin> long
// A long prompt: ids.bin holds n ids (n <= 255); prefill ids[0..n-1) as one chunk (its
// projections on the tensor cores), then step ids[n-1]; logits.bin: FP32 [2][vocab].
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "qwen_forward.hpp"

namespace {

struct Reader {
    FILE* f;
    template <class T>
    std::vector<T> take(size_t n) {
        std::vector<T> v(n);
        if (std::fread(v.data(), sizeof(T), n, f) != n) throw std::runtime_error("short weights file");
        return v;
    }
};

std::vector<void*> g_device;

const uint16_t* upload(const std::vector<uint16_t>& h) {
    void* d = nullptr;
    if (cudaMalloc(&d, h.size() * 2) != cudaSuccess) throw std::runtime_error("cudaMalloc");
    if (cudaMemcpy(d, h.data(), h.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess) throw std::runtime_error("cudaMemcpy");
    g_device.push_back(d);
    return static_cast<const uint16_t*>(d);
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 4) return 2;
    FILE* wf = std::fopen(argv[1], "rb");
    if (!wf) return 3;
    Reader r{wf};
    const std::vector<int32_t> dims = r.take<int32_t>(4);
    const int L = dims[0], H = dims[1], F = dims[2], V = dims[3];
    qattn_host::ForwardWeights w;
    w.hidden = H; w.intermediate = F; w.vocab = V;
    const std::vector<uint16_t> embed = r.take<uint16_t>((size_t)V * H);
    w.embed_host = embed.data();
    w.embed_device = upload(embed);
    const std::vector<float> final_norm = r.take<float>(H);
    w.final_norm = final_norm.data();
    std::vector<std::vector<float>> norms;
    norms.reserve(4 * L);
    for (int l = 0; l < L; ++l) {
        qattn_host::LayerWeights lw;
        norms.push_back(r.take<float>(H)); lw.input_norm = norms.back().data();
        norms.push_back(r.take<float>(H)); lw.post_norm = norms.back().data();
        norms.push_back(r.take<float>(128)); lw.q_norm = norms.back().data();
        norms.push_back(r.take<float>(128)); lw.k_norm = norms.back().data();
        lw.q = upload(r.take<uint16_t>((size_t)2048 * H));
        lw.k = upload(r.take<uint16_t>((size_t)1024 * H));
        lw.v = upload(r.take<uint16_t>((size_t)1024 * H));
        lw.o = upload(r.take<uint16_t>((size_t)H * 2048));
        lw.gate = upload(r.take<uint16_t>((size_t)F * H));
        lw.up = upload(r.take<uint16_t>((size_t)F * H));
        lw.down = upload(r.take<uint16_t>((size_t)H * F));
        w.layers.push_back(lw);
    }
    std::fclose(wf);
    const bool long_prompt = argc > 4 && std::string(argv[4]) == "long";
    FILE* idf = std::fopen(argv[2], "rb");
    if (!idf) return 4;
    std::vector<int32_t> ids(long_prompt ? 255 : 13);
    const size_t got = std::fread(ids.data(), 4, ids.size(), idf);
    std::fclose(idf);
    if (long_prompt) {
        if (got < 2) return 5;
        ids.resize(got);
    } else if (got != ids.size()) {
        return 5;
    }

    qattn_host::Options opt;
    opt.layers = L;
    opt.context = long_prompt ? 256 : 64;
    qattn_host::QwenForward model(w, opt);
    std::vector<float> out;
    auto keep = [&](const std::vector<float>& lg) { out.insert(out.end(), lg.begin(), lg.end()); };
    if (long_prompt) {
        keep(model.prefill(std::vector<int>(ids.begin(), ids.end() - 1)));
        keep(model.step(ids.back()));
        FILE* of = std::fopen(argv[3], "wb");
        if (!of) return 6;
        std::fwrite(out.data(), sizeof(float), out.size(), of);
        std::fclose(of);
        std::printf("position %d\n", model.position());
        for (void* d : g_device) cudaFree(d);
        return 0;
    }
    keep(model.prefill(std::vector<int>(ids.begin(), ids.begin() + 8)));
    keep(model.step(ids[8]));
    keep(model.step(ids[9]));
    keep(model.verify_two(ids[10], ids[11]));
    model.commit_verified(2);
    keep(model.step(ids[12]));
    model.truncate(5);
    keep(model.prefill(std::vector<int>(ids.begin() + 5, ids.begin() + 9)));
    keep(model.step(ids[9]));
    FILE* of = std::fopen(argv[3], "wb");
    if (!of) return 6;
    std::fwrite(out.data(), sizeof(float), out.size(), of);
    std::fclose(of);
    std::printf("position %d\n", model.position());
    for (void* d : g_device) cudaFree(d);
    return 0;
}
