// Prints the ring configuration the launcher picks for each narrow fused tile
// (PickTmem / TmemCfg of fused_tmem_kernel.cuh), one line per (format, BN):
//   <format> <BN> <RSK> <SR> <NRND> <NBR> <INFLIGHT> <GROUPS>
// tests/test_ring_protocol.py checks its Python model's copy of these rules
// against this output.  Host code only: no kernel is launched.
#include <cstdio>
#include "fused_tmem_kernel.cuh"

template <int BN, int FMT>
static void show(const char* name) {
    using C = typename tb::PickTmem<BN, FMT>::Cfg;
    std::printf("%s %d %d %d %d %d %d %d\n", name, BN, C::RSK, C::SR, C::NRND, C::NBR, C::INFLIGHT, C::GROUPS ? 1 : 0);
}

int main() {
    show<16, tb::kE4M3>("E4M3");
    show<64, tb::kE4M3>("E4M3");
    show<128, tb::kE4M3>("E4M3");
    show<16, tb::kE2M1>("E2M1");
    show<64, tb::kE2M1>("E2M1");
    show<128, tb::kE2M1>("E2M1");
    show<16, tb::kBF16>("BF16");
    show<64, tb::kBF16>("BF16");
    show<16, tb::kTF32>("TF32");
    show<64, tb::kTF32>("TF32");
    return 0;
}
