// peer.cuh — the per-rank workspace through which the one-pass kernel of every rank exchanges its
// float64 partial with the other ranks over NVLink (ctb_chain_rows_allsum). Each rank allocates
// one workspace in its own memory (ctb_peer_alloc) and maps every other rank's through CUDA IPC
// (ctb_peer_open); the kernel gets the array of all ranks' workspace addresses.
//
// Slots are double-buffered by the parity of the call's epoch: rank r writes its epoch-e partial
// into slots[e & 1][r] of every rank, and a reader of epoch e accepts a slot only when its epoch
// is exactly e. A rank can be at most one epoch ahead of any other (its call e + 1 cannot finish
// before every rank has published e + 1, which each rank does only after its call e has ended,
// calls of one rank running in stream order), so a slot of parity e & 1 is not overwritten (by
// epoch e + 2) while a slower rank may still be reading its epoch-e value.
#pragma once

#include <cstdint>

namespace ctb {

constexpr int kPeerMaxRanks = 64;
constexpr int kPeerMaxCtas = 4096;
constexpr int kPeerTraceSlots = 64;

// Per-call timestamps (%globaltimer, ns, this GPU's clock), kept for the last kPeerTraceSlots calls
// at trace[epoch % kPeerTraceSlots]: when CTA 0 started, when the first and the last CTA finished
// their rows, and when the exchange completed (or its wait ran out).
enum PeerTrace { kTraceStart = 0, kTraceFirstDone = 1, kTraceLastDone = 2, kTraceExchanged = 3 };

struct alignas(16) PeerSlot {
    double value;    // rank r's partial (written by rank r into every rank's slot r)
    uint64_t epoch;  // the call that wrote it; stored after the value, with release semantics
};

struct alignas(128) PeerWorkspace {
    unsigned ticket;        // CTAs of this rank's launch that have finished (reset by the last one)
    unsigned pad0;
    uint64_t done_epoch;    // the last call whose exchange completed on this rank
    uint64_t failed_epoch;  // the last call whose wait ran out on this rank (0: none)
    uint64_t pad1[13];
    PeerSlot slots[2][kPeerMaxRanks];  // [epoch & 1][writer rank]
    uint64_t trace[kPeerTraceSlots][4];  // PeerTrace timestamps by epoch % kPeerTraceSlots
    double partials[kPeerMaxCtas];       // this rank's per-CTA partials
};

}  // namespace ctb
