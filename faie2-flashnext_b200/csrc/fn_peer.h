// Peer-memory groups: one CUDA-IPC-exported buffer per rank (one process per GPU), every rank's buffer mapped into
// every rank, for kernels that store their results straight into the other GPUs' memory over NVLink and signal
// arrival with release atomics. The buffer layout is the same on every rank.
#pragma once

#include "fn_engine.h"

namespace fn {

// symmetric-buffer layout (bytes)
constexpr size_t PEER_KEY_COUNTERS = 0;     // uint32 [MAX_RANKS]: lm_head key arrivals per source rank
constexpr size_t PEER_MOE_COUNTERS = 256;   // uint32 [MAX_RANKS]: MoE slot-output arrivals per source rank
constexpr size_t PEER_KEYS = 1024;          // uint64 [2][MAX_RANKS][8]: lm_head keys per parity, rank, token
constexpr size_t PEER_MOE = 4096;           // MoE slot outputs (fn_moe_ep.cu)
constexpr size_t PEER_MIN_BYTES = PEER_MOE;

struct PeerGroup {
    int rank = 0, n = 1, dev = 0;
    size_t bytes = 0;
    uint8_t *base[MAX_RANKS] = {};  // every rank's buffer as mapped in this process (base[rank] is this rank's own)
    uint32_t *local_calls = nullptr;  // device counters of this rank: [0] key publishes, [1] key combines, [2..4]
                                      // MoE calls, expected MoE arrivals, MoE combine ticket
    bool mapped[MAX_RANKS] = {};      // base[r] was opened here (closed at free)
};

PeerGroup *peer_group(int g);
// the KeyExchange of a group (lm_head split)
KeyExchange key_exchange(const PeerGroup &pg);

}  // namespace fn
