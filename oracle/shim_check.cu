// Drop-in check of the C++ shim (inferencer-jetson_b200/host/fast_runner.hpp)
// against the reference's own runner, in one program (test infrastructure).
//
// This file #includes the reference's inferencer.cu unmodified (its `main`
// renamed, see oracle/Makefile.ref) and uses the reference's host code the way
// its own main does: GGUF reader, upload, FastRunner construction, forward,
// prefill, gpu.x / gpu.logits / gpu.start_timer / stop_timer / gpu_seconds /
// gpu.calls, FastGPU::matvec and the --compare-prefill traces
// (inferencer.cu:1707-1833, :1855-1889).  The same calls are made on
// ijb_host::FastRunner, the shim over libijb200.so, built from the same GGUF
// object; the program prints one JSON line comparing the two and exits 0.
//
//   shim_check <model.gguf> <use_dp4a 0|1> <token>...
#define main reference_main
#include "inferencer.cu"
#undef main

#include "../inferencer-jetson_b200/host/fast_runner.hpp"

namespace {

std::vector<float> download(const float *dev, int n) {
    std::vector<float> h(n);
    cuda_check(cudaMemcpy(h.data(), dev, n * sizeof(float), cudaMemcpyDeviceToHost), "check download");
    return h;
}

double rel_l2(const std::vector<float> &a, const std::vector<float> &b) {
    double num = 0, den = 0;
    for (size_t i = 0; i < a.size(); ++i) {
        num += (double(a[i]) - b[i]) * (double(a[i]) - b[i]);
        den += double(b[i]) * b[i];
    }
    return std::sqrt(num / (den > 0 ? den : 1));
}

}  // namespace

int main(int argc, char **argv) {
    try {
        if (argc < 4) throw std::runtime_error("usage: shim_check <model.gguf> <use_dp4a> <token>...");
        const bool dp4a = std::atoi(argv[2]) != 0;
        std::vector<int> input;
        for (int i = 3; i < argc; ++i) input.push_back(std::atoi(argv[i]));
        GGUF model(argv[1]);
        model.upload();
        const int context = 64;
        FastRunner ref(model, context, dp4a, dp4a, false, false, 4, 4, 32);
        // the reference caches K/V in fp32 (inferencer.cu:1132); the shim is built with the same format
        ijb_host::FastRunner ours(model, context, dp4a, dp4a, false, false, 4, 4, 32, 0, true);
        if (ours.dim != ref.dim || ours.layers != ref.layers || ours.vocab != ref.vocab)
            throw std::runtime_error("shape fields differ");

        // token by token, timed the way main's decode loop does
        double worst_logits = 0, worst_x = 0;
        int agree = 0;
        for (size_t i = 0; i < input.size(); ++i) {
            ref.gpu.start_timer();
            int a = ref.forward(input[i], static_cast<int>(i), true);
            ref.gpu.stop_timer();
            ours.gpu.start_timer();
            int b = ours.forward(input[i], static_cast<int>(i), true);
            ours.gpu.stop_timer();
            agree += a == b;
            worst_logits = std::max(worst_logits, rel_l2(download(ours.gpu.logits, ours.vocab),
                                                         download(ref.gpu.logits, ref.vocab)));
            worst_x = std::max(worst_x, rel_l2(download(ours.gpu.x, ours.dim), download(ref.gpu.x, ref.dim)));
        }

        // batched prefill of the whole input (FastRunner::prefill)
        ref.reset();
        ours.reset();
        int pa = ref.prefill(input), pb = ours.prefill(input);
        double prefill_logits = rel_l2(download(ours.gpu.logits, ours.vocab), download(ref.gpu.logits, ref.vocab));

        // --compare-prefill's traces on the shim: token-by-token vs batched
        std::vector<std::vector<float>> layers_seq, layers_batch, all_batch;
        std::vector<std::vector<int8_t>> q_seq, q_batch, q_first;
        ours.reset();
        for (size_t i = 0; i < input.size(); ++i) {
            std::vector<std::vector<float>> token_layers;
            ours.forward(input[i], static_cast<int>(i), i + 1 == input.size(), &token_layers,
                         i + 1 == input.size() ? &q_seq : nullptr);
            if (i + 1 == input.size()) layers_seq = token_layers;
        }
        ours.reset();
        ours.prefill(input, &layers_batch, &q_batch, &all_batch, &q_first);
        double trace_diff = 0;
        for (size_t l = 0; l < layers_seq.size(); ++l)
            trace_diff = std::max(trace_diff, rel_l2(layers_batch[l], layers_seq[l]));
        size_t q_same = 0, q_total = 0;
        for (size_t k = 0; k < q_seq.size(); ++k)
            for (size_t j = 0; j < q_seq[k].size(); ++j) {
                q_same += q_seq[k][j] == q_batch[k][j];
                ++q_total;
            }

        // FastGPU::matvec on a model tensor
        const Tensor &wq = model.tensor("blk.0.attn_q.weight");
        float *xin = nullptr, *ya = nullptr, *yb = nullptr;
        cuda_check(cudaMalloc(&xin, ref.dim * sizeof(float)), "alloc");
        cuda_check(cudaMalloc(&ya, ref.dim * sizeof(float)), "alloc");
        cuda_check(cudaMalloc(&yb, ref.dim * sizeof(float)), "alloc");
        cuda_check(cudaMemcpy(xin, ref.gpu.logits, ref.dim * sizeof(float), cudaMemcpyDeviceToDevice), "copy");
        ref.gpu.matvec(wq, xin, ya, ref.dim, ref.dim);
        ours.gpu.matvec(wq, xin, yb, ours.dim, ours.dim);
        cuda_check(cudaDeviceSynchronize(), "sync");
        double matvec_diff = rel_l2(download(yb, ours.dim), download(ya, ref.dim));
        cudaFree(xin);
        cudaFree(ya);
        cudaFree(yb);

        printf("{\"tokens\": %zu, \"forward_agree\": %d, \"forward_logits_rel\": %.3e, \"forward_x_rel\": %.3e, "
               "\"prefill_next\": [%d, %d], \"prefill_logits_rel\": %.3e, \"trace_layers\": %zu, "
               "\"all_layer_trace\": %zu, \"trace_rel\": %.3e, \"quant_trace_vectors\": %zu, "
               "\"quant_trace_same\": %.4f, \"first_quant_vectors\": %zu, \"matvec_rel\": %.3e, "
               "\"gpu_seconds\": [%.6f, %.6f], \"calls\": [%llu, %llu]}\n",
               input.size(), agree, worst_logits, worst_x, pa, pb, prefill_logits, layers_batch.size(),
               all_batch.size(), trace_diff, q_batch.size(), q_total ? double(q_same) / q_total : 0.0,
               q_first.size(), matvec_diff, ref.gpu.gpu_seconds, ours.gpu.gpu_seconds,
               static_cast<unsigned long long>(ref.gpu.calls), ours.gpu.calls);
        return 0;
    } catch (const std::exception &e) {
        std::cerr << "Error: " << e.what() << '\n';
        return 1;
    }
}
