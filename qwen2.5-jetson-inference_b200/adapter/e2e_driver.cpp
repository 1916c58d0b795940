// End-to-end harness: the reference engine (Qwen2Model, reference
// src/qwen2.cpp) driven with token ids, printing one JSON line.  Built twice
// by adapter/Makefile: once against the reference's own Linear kernels and
// once against the b200 kernels through infer_cuda_linear.cpp, so the two
// runs differ only in the Linear layers.
//
//   e2e_driver --model DIR --token-ids 1,2,3 [--backend cuda|cpu]
//              [--precision w16a16|w8a16|fp32] [--linear-kernel custom|cublas]
//              [--new-tokens 128] [--warmup 5] [--repeat 20]
//              [--max-seq-len 256] [--logits-out FILE]
//              [--force-tokens CSV]
//
// Output: generated token ids (greedy, no EOS stop, as the reference's
// benchmark mode runs), per-repeat TTFT / decode tok/s / TPOT (the
// reference's definitions, include/infer/qwen2.hpp:29-33), and optionally
// the FP32 logits after prefill (for the cosine check of
// tests/test_qwen2.cpp:490-511).  With --force-tokens the driver also runs
// one teacher-forced pass: after the prefill it feeds the given tokens
// (another engine's greedy output) to decode_next and records its own argmax
// and the gap between its two largest logits at every step, which tells a
// near-tie apart from a real disagreement.
#include <algorithm>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "infer/qwen2.hpp"

namespace {

std::string arg(int argc, char** argv, const std::string& key,
                const std::string& fallback = "") {
  for (int i = 1; i + 1 < argc; ++i) {
    if (key == argv[i]) return argv[i + 1];
  }
  return fallback;
}

std::vector<int> parse_ids(const std::string& csv) {
  std::vector<int> ids;
  std::stringstream ss(csv);
  std::string item;
  while (std::getline(ss, item, ',')) {
    if (!item.empty()) ids.push_back(std::stoi(item));
  }
  return ids;
}

template <class T>
std::string json_list(const std::vector<T>& v) {
  std::ostringstream os;
  os << '[';
  for (size_t i = 0; i < v.size(); ++i) os << (i ? "," : "") << v[i];
  os << ']';
  return os.str();
}

}  // namespace

// Present when the binary links libb200linear.so (e2e_b200), absent in
// e2e_reference: the W8A16 prefill's BF16 weight buffer is reserved once at
// start-up, as the reference engine allocates its own workspaces at load.
extern "C" int b200_gemm_reserve_scratch(size_t bytes) __attribute__((weak));

int main(int argc, char** argv) {
  try {
    infer::RuntimeOptions opt;
    const std::string backend = arg(argc, argv, "--backend", "cuda");
    opt.backend = backend == "cpu" ? infer::Device::kCpu : infer::Device::kCuda;
    const std::string prec = arg(argc, argv, "--precision",
                                 backend == "cpu" ? "fp32" : "w16a16");
    opt.precision = prec == "fp32"   ? infer::Precision::kFloat32
                    : prec == "w8a16" ? infer::Precision::kW8A16
                                      : infer::Precision::kW16A16;
    opt.linear_kernel = arg(argc, argv, "--linear-kernel", "custom") == "cublas"
                            ? infer::LinearKernel::kCublas
                            : infer::LinearKernel::kCustom;
    opt.max_sequence_length = std::stoi(arg(argc, argv, "--max-seq-len", "256"));
    const auto prompt = parse_ids(arg(argc, argv, "--token-ids"));
    const int new_tokens = std::stoi(arg(argc, argv, "--new-tokens", "128"));
    const int warmup = std::stoi(arg(argc, argv, "--warmup", "5"));
    const int repeat = std::stoi(arg(argc, argv, "--repeat", "20"));
    const std::string logits_out = arg(argc, argv, "--logits-out");
    if (prompt.empty()) throw infer::Error("--token-ids is required");

    infer::Qwen2Model model(arg(argc, argv, "--model"), opt);
    if (b200_gemm_reserve_scratch != nullptr && opt.backend == infer::Device::kCuda &&
        opt.precision == infer::Precision::kW8A16) {
      if (b200_gemm_reserve_scratch(0) != 0) throw infer::Error("b200_gemm_reserve_scratch");
    }
    if (!logits_out.empty()) {
      model.reset();
      model.prefill(prompt);
      const auto logits = model.last_logits_host();
      std::ofstream f(logits_out, std::ios::binary);
      f.write(reinterpret_cast<const char*>(logits.data()),
              std::streamsize(logits.size() * sizeof(float)));
    }
    std::vector<int> forced_argmax;
    std::vector<float> forced_gap;
    const auto forced = parse_ids(arg(argc, argv, "--force-tokens"));
    if (!forced.empty()) {
      auto gap = [&]() {
        const auto l = model.last_logits_host();
        float a = -1e30f, b = -1e30f;
        for (float v : l) {
          if (v > a) { b = a; a = v; } else if (v > b) { b = v; }
        }
        return a - b;
      };
      model.reset();
      forced_argmax.push_back(model.prefill(prompt));
      forced_gap.push_back(gap());
      for (size_t j = 0; j + 1 < forced.size(); ++j) {
        forced_argmax.push_back(model.decode_next(forced[j]));
        forced_gap.push_back(gap());
      }
    }
    for (int i = 0; i < warmup; ++i) model.generate(prompt, new_tokens, false);
    std::vector<int> tokens;
    std::vector<double> ttft, decode, tpot;
    for (int i = 0; i < std::max(1, repeat); ++i) {
      const auto r = model.generate(prompt, new_tokens, false);
      if (i == 0) tokens = r.tokens;
      if (r.tokens != tokens) throw infer::Error("generation is not deterministic");
      ttft.push_back(r.stats.ttft_ms);
      decode.push_back(r.stats.decode_tokens_per_second());
      tpot.push_back(r.stats.generated_tokens > 1
                         ? r.stats.decode_ms / (r.stats.generated_tokens - 1)
                         : 0.0);
    }
    std::cout << "{\"tokens\":" << json_list(tokens)
              << ",\"ttft_ms\":" << json_list(ttft)
              << ",\"decode_tok_s\":" << json_list(decode)
              << ",\"tpot_ms\":" << json_list(tpot)
              << ",\"forced_argmax\":" << json_list(forced_argmax)
              << ",\"forced_gap\":" << json_list(forced_gap)
              << ",\"device_weight_bytes\":" << model.device_weight_bytes()
              << "}" << std::endl;
  } catch (const std::exception& e) {
    std::cerr << "error: " << e.what() << std::endl;
    return 2;
  }
  return 0;
}
