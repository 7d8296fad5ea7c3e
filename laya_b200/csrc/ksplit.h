// ksplit.h — how many K chunks an accumulating bf16 product is split into (host code, no CUDA dependency).
//
// Few output tiles over a long K (weight gradients dW += dYᵀ·X: K = tokens) leave most SMs idle, so an accumulating
// output splits K into chunks of at least 4 k-blocks whose partial tiles reduce-add into it. The chunk count
// minimises (rounds of work units over the SMs) × (k-blocks per unit + one for the unit's epilogue), so the last
// round is not left mostly idle: 54 tiles over 320 k-blocks on 148 SMs take 8 chunks (432 units, 3 rounds nearly
// full) rather than 6 (324 units, 3 rounds with the last a fifth full).
#pragma once

namespace laya {
namespace bf {

// Every returned chunk count leaves every chunk non-empty: with kchunk = ceil(kblocks / ks), the last chunk starts
// below kblocks.
inline int choose_ksplit(int tiles, int kblocks, int nsm) {
    if (tiles <= 0 || kblocks <= 0 || nsm <= 0 || tiles >= nsm) return 1;
    int ksplit = 1;
    long best = -1;
    const int most = kblocks / 4 > 1 ? kblocks / 4 : 1;
    for (int want = 1; want <= most; ++want) {
        const int kchunk = (kblocks + want - 1) / want;
        const int ks = (kblocks + kchunk - 1) / kchunk;
        const long rounds = (static_cast<long>(tiles) * ks + nsm - 1) / nsm;
        const long cost = rounds * (kchunk + 1);
        if (best < 0 || cost < best) { best = cost; ksplit = ks; }
    }
    return ksplit;
}

}  // namespace bf
}  // namespace laya
