// Data-parallel FT row exchange over peer memory (exchange.cu): flag waits
// and signals between ranks, the owners' Ranger + broadcast of their shard.
#pragma once

#include "common.cuh"

namespace bou {

constexpr int kExchangeMaxRanks = 8;

// Every rank's flag words (device addresses, peers' through CUDA IPC).
struct PeerFlags {
    int* p[kExchangeMaxRanks];
};

// Stores `epoch` into flags[index] of every rank, after a system-scope fence
// (the data written before on this stream is visible to the peers first).
int launch_exchange_signal(BulletOuCudaCppContext* ctx, const PeerFlags& flags, int world, size_t index, int epoch);

// Copies src[0, len) into slot `rank` (of len floats) of every rank's buffer
// dst[r], then fences at system scope.
struct PeerBuffers {
    float* p[kExchangeMaxRanks];
};
int launch_exchange_scatter(BulletOuCudaCppContext* ctx, const float* src, size_t len, const PeerBuffers& dst,
                            int world, int rank);

// One thread waits until flags[0, count) all hold at least `epoch`; after
// about 2 s it stores 1 + the index of the flag it waited for into *error and
// returns.
int launch_exchange_wait(BulletOuCudaCppContext* ctx, const int* flags, int count, int epoch, int* error);

}  // namespace bou
