// peer.cuh — the per-rank workspace through which the one-pass kernel of every rank exchanges its
// float64 partial with the other ranks over NVLink (ctb_chain_rows_allsum). Each rank allocates
// one workspace in its own memory (ctb_peer_alloc) and maps every other rank's through CUDA IPC
// (ctb_peer_open); the kernel gets the array of all ranks' workspace addresses.
#pragma once

#include <cstdint>

namespace ctb {

constexpr int kPeerMaxRanks = 64;
constexpr int kPeerMaxCtas = 4096;

struct alignas(16) PeerSlot {
    double value;    // rank r's partial (written by rank r into every rank's slot r)
    uint64_t epoch;  // the call that wrote it; stored after the value, with release semantics
};

struct alignas(128) PeerWorkspace {
    unsigned ticket;  // CTAs of this rank's launch that have finished (reset by the last one)
    unsigned pad[31];
    PeerSlot slots[kPeerMaxRanks];
    double partials[kPeerMaxCtas];  // this rank's per-CTA partials
};

}  // namespace ctb
