// Tuning-harness driver for the B200 attention engine.
//
// Drop-in for tuning/attn_test.cu of the reference: the harness
// (tuning/benchmark_run_attn.py) rewrites the `constexpr` lines in main()
// below (benchmark_run_attn.py:155-170), compiles this file with
//   nvcc -std=c++17 -arch=sm_100a -O3 <file> -o <exe> -lcuda -Xptxas=-v
// and parses the last "B, H, S, D, BM, BN, avg_ms, tflops" line.  Pass
// --source pointing here and --build-dir inside this directory (for example
// attnprofile_b200/harness/build, up to two levels below) so the generated
// copy finds its includes.
#if __has_include("attn_harness.cuh")
#include "attn_harness.cuh"
#elif __has_include("../attn_harness.cuh")
#include "../attn_harness.cuh"
#elif __has_include("../../attn_harness.cuh")
#include "../../attn_harness.cuh"
#else
#error "compile from attnprofile_b200/harness or a subdirectory of it (use --build-dir there)"
#endif

// nvcc -std=c++17 -arch=sm_100a -O3 attn_test.cu -o attn_test -lcuda -Xptxas=-v
int main() {
    constexpr int BM = 256;
    constexpr int BN = 128;
    constexpr int B = 1;
    constexpr int H = 16;
    constexpr int S = 4096;
    constexpr int D = 128;

    constexpr int NUM_SMEM = 2;
    constexpr uint32_t PRODUCER_REG_DEALLOC = 24;
    constexpr uint32_t CONSUMER_REG_ALLOC = 240;
    constexpr int P_SMEM_K_TILES = 0;
    constexpr int KERNEL_IDX = 1;
    constexpr int NUM_THREADS = 384;

    auto *kernel = runAttn<
        B, H, S, D, BM, BN, NUM_SMEM,
        PRODUCER_REG_DEALLOC, CONSUMER_REG_ALLOC,
        P_SMEM_K_TILES, KERNEL_IDX, NUM_THREADS>;
    benchmark_attn<B, H, S, D, BM, BN>(kernel);
    return 0;
}
