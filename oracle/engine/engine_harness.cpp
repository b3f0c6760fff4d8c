// engine_harness.cpp — drives the Genllm engine itself (its GGUF loader,
// graph builder, GraphScheduler, MemoryManager and Executor, compiled from the
// Genllm sources by oracle/engine/Makefile) through a greedy decode, the
// config-2 workload of the paged KV-cache path: a prompt of seeded random ids
// prefilled with Executor::append_tokens in chunks (src/core/executor.cpp:
// 237-247), then decode_step (:227-236) with the argmax of the last logits row
// taken here (the engine's own sample() draws from a random-seeded top-p,
// :291-340, and sample_argmax is private).
//
// Test infrastructure only. The same source links into three engines: the
// CPU engine, the CUDA engine with Genllm's own paged attention, and the CUDA
// engine whose ops::PagedAttentionImpl<Device::CUDA> is this repository's
// drop-in adapter (genllm_b200/adapter/paged_attention_cuda.cpp).
//
// Usage: engine_harness GGUF PROMPT_LEN DECODE_STEPS CHUNK SEED OUT [FORCED|random]
//   OUT receives, per predicted position (after the prefill, then after each
//   decode step): int32 argmax, float top-1, float top-2 logit, and the full
//   logits row (bf16) at the positions listed in kDumpSteps. FORCED (int32
//   ids) replaces the argmax as the next input (teacher forcing); "random"
//   feeds seeded random ids instead, so that every engine sees the same
//   inputs and its predictions can be compared position by position.
#include <chrono>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <print>
#include <string>
#include <vector>

#include "backend/backend.h"
#include "core/executor.h"
#include "core/gguf_parser.h"
#include "core/graph.h"
#include "model/model.h"
#ifdef BACKEND_CUDA
#include <cuda_runtime.h>
#endif

namespace {

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

float bf16_to_f32(uint16_t b) {
    uint32_t u = static_cast<uint32_t>(b) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

struct Row {
    int32_t argmax;
    float top1, top2;
};

// The last position's logits row, copied to the host if the engine left it
// on a device.
std::vector<uint16_t> last_row(const ComputeGraph& g, size_t vocab) {
    const Tensor* t = g.get_external_outputs()[0];
    const int64_t pos = t->dims[1] - 1;
    std::vector<uint16_t> row(vocab);
    const auto* src = static_cast<const uint16_t*>(t->data) + pos * vocab;
#ifdef BACKEND_CUDA
    if (t->device != Device::CPU) {
        cudaMemcpy(row.data(), src, vocab * 2, cudaMemcpyDeviceToHost);
        return row;
    }
#endif
    std::memcpy(row.data(), src, vocab * 2);
    return row;
}

Row summarize(const std::vector<uint16_t>& row) {
    Row r{0, -INFINITY, -INFINITY};
    for (size_t i = 0; i < row.size(); ++i) {
        const float v = bf16_to_f32(row[i]);
        if (v > r.top1) {
            r.top2 = r.top1;
            r.top1 = v;
            r.argmax = static_cast<int32_t>(i);
        } else if (v > r.top2) {
            r.top2 = v;
        }
    }
    return r;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 7) {
        std::fprintf(stderr, "usage: %s GGUF PROMPT_LEN DECODE_STEPS CHUNK SEED OUT [FORCED]\n", argv[0]);
        return 2;
    }
    const std::string path = argv[1];
    const int prompt_len = std::stoi(argv[2]);
    const int steps = std::stoi(argv[3]);
    const int chunk = std::stoi(argv[4]);
    const uint64_t seed = std::stoull(argv[5]);
    const std::string out_path = argv[6];
    std::vector<int32_t> forced;
    const bool random_inputs = argc > 7 && std::string(argv[7]) == "random";
    if (argc > 7 && !random_inputs) {
        std::ifstream f(argv[7], std::ios::binary);
        int32_t v;
        while (f.read(reinterpret_cast<char*>(&v), 4)) forced.push_back(v);
    }
    const std::vector<int> dump_steps = {0, 1, steps / 2, steps};

    GGUFParser parser(path);
    std::unique_ptr<ModelBase> model = ModelFactory::CreateFromGGUF(parser.info());
    auto graph = model->build_graph(parser.info());
    GraphScheduler::Config cfg{.vocab_size = model->vocab_size(),
                               .max_seq_len = prompt_len + steps + 16,
                               .top_p = 1.0f,
                               .temperature = 1.0f,
                               .memory_headroom = 0.1f,
                               .kv_cache_pool_factor = 1.05f,
                               .activation_pool_factor = 1.05f};
    GraphScheduler scheduler(std::move(graph), cfg);
    scheduler.schedule(DeviceManager::instance().get_devices());
    scheduler.mmanager()->load_weights(parser, scheduler.graph());
    Executor ex(scheduler);
    const size_t vocab = static_cast<size_t>(model->vocab_size());

    // Prompt: seeded ids (64-bit LCG, high bits), uniform over the vocabulary.
    std::vector<int32_t> prompt(prompt_len);
    uint64_t s = seed * 6364136223846793005ull + 1442695040888963407ull;
    auto next_id = [&] {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        return static_cast<int32_t>((s >> 33) % vocab);
    };
    for (auto& id : prompt) id = next_id();
    if (random_inputs)  // the decode inputs continue the same seeded sequence
        for (int i = 0; i < steps; ++i) forced.push_back(next_id());

    std::ofstream out(out_path, std::ios::binary);
    std::vector<int32_t> tokens;
    const double t0 = now_s();
    for (int p = 0; p < prompt_len; p += chunk) {
        std::vector<int32_t> c(prompt.begin() + p, prompt.begin() + std::min(prompt_len, p + chunk));
        ex.append_tokens(c);
    }
    const double t1 = now_s();
    double t_decode = 0.0;
    for (int i = 0; i <= steps; ++i) {
        const std::vector<uint16_t> row = last_row(scheduler.graph(), vocab);
        const Row r = summarize(row);
        out.write(reinterpret_cast<const char*>(&r), sizeof(r));
        for (int d : dump_steps)
            if (d == i) out.write(reinterpret_cast<const char*>(row.data()), row.size() * 2);
        if (i == steps) break;
        const int32_t next = i < static_cast<int>(forced.size()) ? forced[i] : r.argmax;
        tokens.push_back(r.argmax);
        const double a = now_s();
        ex.decode_step(next);
        t_decode += now_s() - a;
    }
    std::print("{{\"prompt_len\": {}, \"steps\": {}, \"prefill_s\": {:.4f}, \"decode_s\": {:.4f}, "
               "\"decode_tok_s\": {:.3f}, \"tokens\": [",
               prompt_len, steps, t1 - t0, t_decode, steps / t_decode);
    for (size_t i = 0; i < tokens.size(); ++i) std::print("{}{}", i ? ", " : "", tokens[i]);
    std::println("]}}");
    return 0;
}
