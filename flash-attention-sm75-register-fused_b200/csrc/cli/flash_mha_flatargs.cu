// flash_mha_flatargs — full (non-causal) attention CLI, d = 64.
// Command line and stdout contract of the reference tool
// flash-attention-sm75-fused/src/flash_mha_flatargs.cu:652-691; the kernel is
// the sm_100a forward behind flatargs_launch() in libfa_b200.so.  Any N is
// accepted (the reference padded N to a multiple of 16).
#include "cli_common.h"

static void run_case(int B, int H, int N, bool do_val, int outer, int inner, bool header) {
  const float scale = 1.f / std::sqrt((float)cli::kD);
  const size_t total = (size_t)B * H * N * cli::kD;
  const double flops = (double)B * H * 4.0 * N * N * cli::kD;
  if (header) {
    cli::print_device();
    std::printf("\n=== flash_mha_flatargs ===\n");
    std::printf("B=%d H=%d N_req=%d N_pad=%d d=%d\n", B, H, N, N, cli::kD);
    std::printf("Grid = %d CTAs (2 x 128-row Q tiles each)\n\n", B * H * ((N + 255) / 256));
  }
  cli::Buffers buf(total);
  std::vector<__half> hq, hk, hv;
  cli::fill_inputs(buf, hq, hk, hv);
  auto launch = [&]() {
    cli::check_fa(flatargs_launch(buf.q, buf.k, buf.v, buf.o, B, H, N, scale, nullptr),
                  "flatargs_launch");
  };
  if (do_val) {
    std::vector<float> ref(total);
    std::printf("[1/3] CPU reference... ");
    std::fflush(stdout);
    cli::cpu_attention(hq, hk, hv, ref, B, H, N, cli::kD, scale, false);
    std::printf("OK\n[2/3] GPU kernel... ");
    launch();
    cli::check(cudaDeviceSynchronize(), "sync");
    std::printf("OK\n[3/3] Validation...\n");
    std::vector<__half> out(total);
    cli::check(cudaMemcpy(out.data(), buf.o, total * sizeof(__half), cudaMemcpyDeviceToHost), "D2H");
    const bool ok = cli::validate(out, ref, B, H, N, cli::kD, "FULL");
    std::printf("  Result: %s\n\n", ok ? "PASS" : "FAIL");
  }
  const cli::Stats st = cli::bench(launch, outer, inner);
  auto tf = [&](double ms) { return flops / (ms * 1e-3) / 1e12; };
  if (header) {
    std::printf("=== Benchmark (outer=%d inner=%d) ===\n", outer, inner);
    std::printf("  %-12s %-10s %-10s %-10s\n", "metric", "min", "median", "max");
    std::printf("  %-12s %-10.4f %-10.4f %-10.4f\n", "ms", st.min_ms, st.med_ms, st.max_ms);
    std::printf("  %-12s %-10.4f %-10.4f %-10.4f\n\n", "TFLOPS", tf(st.max_ms), tf(st.med_ms),
                tf(st.min_ms));
  } else {
    std::printf("%-5d %-5d %-6d | %-8.4f %-8.4f %-8.4f | %-8.2f %-8.2f %-8.2f\n", B, H, N,
                st.min_ms, st.med_ms, st.max_ms, tf(st.max_ms), tf(st.med_ms), tf(st.min_ms));
  }
}

int main(int argc, char** argv) {
  std::printf("flash_mha_flatargs — B200 sm_100a (tcgen05)  d=64\n\n");
  if (argc == 1) {
    run_case(1, 2, 64, true, 5, 100, true);
    run_case(1, 4, 128, true, 5, 100, true);
    std::printf("=== Sweep flash_mha_flatargs (d=64) ===\n");
    std::printf("%-5s %-5s %-6s | %-26s | %-26s\n", "B", "H", "N", "latency ms (min med max)",
                "TFLOPS (max med min)");
    const int cfgs[][3] = {{1, 1, 256},  {1, 1, 512},  {1, 1, 1024}, {1, 8, 256},
                           {4, 8, 256},  {8, 8, 256},  {4, 12, 512}, {4, 12, 1024},
                           {8, 12, 512}, {1, 16, 2048}, {4, 8, 2048}};
    for (auto& c : cfgs) run_case(c[0], c[1], c[2], false, 7, 100, false);
    return 0;
  }
  const int B = std::atoi(argv[1]);
  const int H = argc > 2 ? std::atoi(argv[2]) : 1;
  const int N = argc > 3 ? std::atoi(argv[3]) : 256;
  const int outer = argc > 4 ? std::atoi(argv[4]) : 7;
  const int inner = argc > 5 ? std::atoi(argv[5]) : 100;
  if (B <= 0 || H <= 0 || N <= 0) {
    std::fprintf(stderr, "usage: %s [B H N [outer [inner]]]\n", argv[0]);
    return 2;
  }
  const bool do_val = (double)B * H * N * N * cli::kD < 3e8;
  run_case(B, H, N, do_val, outer, inner, true);
  return 0;
}
