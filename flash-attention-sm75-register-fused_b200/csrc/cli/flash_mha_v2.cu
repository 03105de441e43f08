// flash_mha_v2 — full and causal attention CLI, d = 64.
// Command line and stdout contract of the reference tool
// flash-attention-sm75-fused/src/flash_mha_v2.cu:790-816 (lines starting with
// "FULL" / "CAUSAL" followed by min/median/max ms, parsed by
// benchmark_sdpa_final.py:126-141); causal TFLOPS count half of 4*B*H*N^2*d.
// The kernel is the sm_100a forward behind launch_v2() in libfa_b200.so.
#include "cli_common.h"

static void run_case(int B, int H, int N, bool do_val, int outer, int inner, bool header) {
  const float scale = 1.f / std::sqrt((float)cli::kD);
  const size_t total = (size_t)B * H * N * cli::kD;
  const double flops_full = (double)B * H * 4.0 * N * N * cli::kD;
  const double flops_causal = flops_full * 0.5;
  if (header) {
    cli::print_device();
    std::printf("\n=== flash_v2  B=%d H=%d N=%d d=64 ===\n\n", B, H, N);
  }
  cli::Buffers buf(total);
  std::vector<__half> hq, hk, hv;
  cli::fill_inputs(buf, hq, hk, hv);
  auto launch = [&](int mode) {
    cli::check_fa(launch_v2(buf.q, buf.k, buf.v, buf.o, B, H, N, scale, mode, nullptr), "launch_v2");
  };
  if (do_val) {
    std::vector<float> ref(total);
    std::vector<__half> out(total);
    for (int mode = 0; mode < 2; ++mode) {
      std::printf("[ref] CPU %s... ", mode ? "causal" : "full");
      std::fflush(stdout);
      cli::cpu_attention(hq, hk, hv, ref, B, H, N, cli::kD, scale, mode == 1);
      std::printf("OK\n");
      launch(mode);
      cli::check(cudaDeviceSynchronize(), "sync");
      cli::check(cudaMemcpy(out.data(), buf.o, total * sizeof(__half), cudaMemcpyDeviceToHost),
                 "D2H");
      cli::validate(out, ref, B, H, N, cli::kD, mode ? "CAUSAL " : "FULL   ");
    }
    std::printf("\n");
  }
  const cli::Stats bf = cli::bench([&]() { launch(0); }, outer, inner);
  const cli::Stats bc = cli::bench([&]() { launch(1); }, outer, inner);
  auto tff = [&](double ms) { return flops_full / (ms * 1e-3) / 1e12; };
  auto tfc = [&](double ms) { return flops_causal / (ms * 1e-3) / 1e12; };
  if (header) {
    std::printf("%-10s %-10s %-10s %-10s %-10s %-10s\n", "", "min_ms", "med_ms", "max_ms",
                "TFLOPS_hi", "TFLOPS_med");
    std::printf("%-10s %-10.4f %-10.4f %-10.4f %-10.4f %-10.4f\n", "FULL", bf.min_ms, bf.med_ms,
                bf.max_ms, tff(bf.min_ms), tff(bf.med_ms));
    std::printf("%-10s %-10.4f %-10.4f %-10.4f %-10.4f %-10.4f\n", "CAUSAL", bc.min_ms,
                bc.med_ms, bc.max_ms, tfc(bc.min_ms), tfc(bc.med_ms));
    std::printf("\n  Speedup causal/full (latency): %.3fx\n\n", bf.med_ms / bc.med_ms);
  } else {
    std::printf("%-5d %-5d %-6d | %-8.4f %-8.2f | %-8.4f %-8.2f | %-6.2fx\n", B, H, N, bf.med_ms,
                tff(bf.med_ms), bc.med_ms, tfc(bc.med_ms), bf.med_ms / bc.med_ms);
  }
}

int main(int argc, char** argv) {
  std::printf("flash_v2 — B200 sm_100a (tcgen05)  d=64  full + causal\n\n");
  if (argc == 1) {
    run_case(1, 2, 64, true, 5, 100, true);
    run_case(1, 4, 128, true, 5, 100, true);
    std::printf("%-5s %-5s %-6s | %-17s | %-17s | %-7s\n", "B", "H", "N", "FULL ms TFLOPS",
                "CAUSAL ms TFLOPS", "lat-spd");
    const int cfgs[][3] = {{1, 8, 256}, {4, 12, 512}, {4, 12, 1024}, {8, 12, 512},
                           {1, 16, 2048}, {4, 8, 2048}};
    for (auto& c : cfgs) run_case(c[0], c[1], c[2], false, 7, 100, false);
    return 0;
  }
  if (argc < 4) {
    std::fprintf(stderr, "usage: %s [B H N [outer [inner]]]\n", argv[0]);
    return 2;
  }
  const int B = std::atoi(argv[1]);
  const int H = std::atoi(argv[2]);
  const int N = std::atoi(argv[3]);
  const int outer = argc > 4 ? std::atoi(argv[4]) : 7;
  const int inner = argc > 5 ? std::atoi(argv[5]) : 100;
  if (B <= 0 || H <= 0 || N <= 0) {
    std::fprintf(stderr, "usage: %s [B H N [outer [inner]]]\n", argv[0]);
    return 2;
  }
  const bool val = (double)B * H * N * N * cli::kD < 3e8;
  run_case(B, H, N, val, outer, inner, true);
  return 0;
}
