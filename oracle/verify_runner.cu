// verify_runner.cu -- the reference's own correctness entry, verify_attn
// (tuning/utils.cuh:73-244), with the B200 engine's runAttn<...> as its
// AttnRunner (tuning/utils.cuh:71), the call the reference's driver makes
// (commented out at tuning/attn_test.cu:1719).
//
// TEST INFRASTRUCTURE ONLY (builds oracle/_ref/verify_runner, never shipped).
// utils.cuh is compiled from where it lies in the reference checkout (the
// Makefile puts its tuning/ directory on the include path; nothing is
// copied).  verify_attn draws its mt19937(42) inputs, runs our kernel on a
// B200, computes its own CPU output and prints
//   [D] hO attention max_abs_diff=... mismatches(abs>0.0500)=...
// which tests/test_gpu_ref_verify.py parses.  Its `prop.major < 9` guard
// passes on a B200 (major 10).
//
//   verify_runner <case>    case 0..5, see the switch below; prints the case
//                           line "case B H S D BM BN" then verify_attn's lines
#include "utils.cuh"

#include "../attnprofile_b200/harness/attn_runner.cuh"

#include <cstdio>
#include <cstdlib>

namespace {
template <int B, int H, int S, int D, int BM, int BN>
void run_case(int idx) {
  std::printf("case %d: B=%d H=%d S=%d D=%d BM=%d BN=%d\n", idx, B, H, S, D, BM, BN);
  std::fflush(stdout);
  // Hopper-only knobs of runAttn (NUM_SMEM, register split, P tiles, kernel
  // index, threads) at the reference driver's defaults (tuning/attn_test.cu:1696-1710).
  verify_attn<B, H, S, D, BM, BN>(runAttn<B, H, S, D, BM, BN, 2, 24, 240, 0, 1, 384>);
  std::fflush(stdout);
}
}  // namespace

int main(int argc, char** argv) {
  const int c = argc > 1 ? std::atoi(argv[1]) : 0;
  switch (c) {
    case 0: run_case<1, 1, 512, 128, 256, 128>(0); break;   // the C1 shape, default tile
    case 1: run_case<1, 1, 512, 128, 128, 64>(1); break;    // one Q tile, narrow key tiles
    case 2: run_case<1, 2, 1000, 128, 256, 128>(2); break;  // ragged: SQO 1024, SKV 1024
    case 3: run_case<2, 2, 300, 64, 256, 96>(3); break;     // D = 64, ragged, padded layout
    // D = 64 tiles that only the tuning harness builds (wide key tiles, one S
    // buffer per Q tile): the reference's D = 64 sweep at BM = 256 reaches them.
    case 4: run_case<1, 2, 1000, 64, 256, 160>(4); break;
    case 5: run_case<1, 2, 1000, 64, 256, 192>(5); break;
    default:
      std::fprintf(stderr, "usage: verify_runner <0..5>\n");
      return 2;
  }
  return 0;
}
