// Prints the ring configurations the launcher picks, one line each:
//   TMEM <format> <BN> <RSK> <SR> <NRND> <NBR> <INFLIGHT> <GROUPS>
//        the narrow few-token kernel (PickTmem / TmemCfg, fused_tmem_kernel.cuh)
//   PAIR <format> <RK> <S> <SA> <DK>
//        the fused SM-pair kernel (PickFusedPair / FusedPairCfg, fused_pair_kernel.cuh)
// tests/test_ring_protocol.py and tests/test_pair_protocol.py check their
// Python models' copies of these rules against this output.  Host code only:
// no kernel is launched.
#include <cstdio>
#include "fused_pair_kernel.cuh"
#include "fused_tmem_kernel.cuh"

template <int BN, int FMT>
static void tmem(const char* name) {
    using C = typename tb::PickTmem<BN, FMT>::Cfg;
    std::printf("TMEM %s %d %d %d %d %d %d %d\n", name, BN, C::RSK, C::SR, C::NRND, C::NBR, C::INFLIGHT,
                C::GROUPS ? 1 : 0);
}

template <int FMT>
static void pair(const char* name) {
    using C = typename tb::PickFusedPair<FMT>::Cfg;
    std::printf("PAIR %s %d %d %d %d\n", name, C::RK, C::S, C::SA, C::DK);
}

int main() {
    tmem<16, tb::kE4M3>("E4M3");
    tmem<64, tb::kE4M3>("E4M3");
    tmem<128, tb::kE4M3>("E4M3");
    tmem<16, tb::kE2M1>("E2M1");
    tmem<64, tb::kE2M1>("E2M1");
    tmem<128, tb::kE2M1>("E2M1");
    tmem<16, tb::kBF16>("BF16");
    tmem<64, tb::kBF16>("BF16");
    tmem<16, tb::kTF32>("TF32");
    tmem<64, tb::kTF32>("TF32");
    pair<tb::kE4M3>("E4M3");
    pair<tb::kE2M1>("E2M1");
    pair<tb::kBF16>("BF16");
    pair<tb::kTF32>("TF32");
    return 0;
}
