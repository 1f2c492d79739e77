// The per-expert count all-gather over peer memory, shared by kb_ep_counts_allgather
// (ep_peer.cu) and the fused form inside the router + maps tile kernel (routing.cu,
// kb_router_maps_allgather), and the layout of the control words and count slots at the start
// of every rank's expert-parallel exchange buffer.
//
// A rank's counts travel as 64-bit words (tag << 32 | count) into slot (tag & 1) of row
// [sender] of every rank's buffer; one word carries its own validity, so the receiver polls
// the words themselves.  The tag is the call's epoch (completed calls + 1, never 0), kept in
// the receiver's own control word.  Slot reuse is safe: rank p writes slot s again two calls
// later, which needs this rank's row of the call in between, which this rank sends only after
// it has read slot s.
#pragma once

#include "kb_common.cuh"

namespace kb {

constexpr int kEpMaxRanks = KB_MAX_RANKS;
// Control words (byte offsets).  Epochs and tickets are written only by the owning rank; the
// arrival counters [kEpMaxRanks] are incremented by the peers.
constexpr size_t kEpErr = 0;            // error word (KB_WS_TIMEOUT / KB_WS_CAPACITY), sticky
constexpr size_t kEpCountEpoch = 4;     // completed count all-gathers
constexpr size_t kEpDispEpoch = 8;      // completed kb_ep_dispatch calls
constexpr size_t kEpCombEpoch = 12;     // completed kb_ep_combine calls
constexpr size_t kEpDispTicket = 16;    // CTAs of the running dispatch that are done sending
constexpr size_t kEpCombTicket = 20;    // CTAs of the running combine send that are done
constexpr size_t kEpFinTicket = 24;     // CTAs of the running combine finalize that are done
constexpr size_t kEpBarEpoch = 28;      // completed kb_ep_barrier calls
constexpr size_t kEpDispArrive = 128;   // [q]: dispatches rank q has completed into this buffer
constexpr size_t kEpCombArrive = 256;   // [q]: combines owner q has completed into this buffer
constexpr size_t kEpBarArrive = 384;    // [q]: barriers rank q has entered
constexpr size_t kEpCountsOff = 512;    // uint64 [2][kEpMaxRanks][E] tagged count rows
constexpr long long kEpSpin = 10000000; // polls before a peer wait gives up (~10 s)

// The count all-gather of one call: every rank's mapped buffer, the output, this rank.
struct CountPush {
    char* buf[kEpMaxRanks];
    int32_t* gathered;     // int32 [world][E]
    int world, rank, E;    // world == 0: no exchange
    long long spin;
    int fused;             // host only: set when the tile kernel took the exchange
};

__device__ __forceinline__ unsigned ep_ld_volatile(const unsigned* p) {
    return *reinterpret_cast<const volatile unsigned*>(p);
}
__device__ __forceinline__ unsigned long long ep_ld_relaxed_sys_u64(const void* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ep_exch_relaxed_sys_u64(void* p, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.relaxed.sys.global.exch.b64 %0, [%1], %2;"
                 : "=l"(old) : "l"(p), "l"(v) : "memory");
    (void)old;
}

// This call's tag (read before the call's own epoch update).
__device__ __forceinline__ unsigned count_push_tag(const CountPush& cp) {
    const unsigned t = ep_ld_volatile(reinterpret_cast<const unsigned*>(cp.buf[cp.rank] + kEpCountEpoch)) + 1u;
    return t ? t : 1u;
}
__device__ __forceinline__ char* count_slot(const CountPush& cp, int q, unsigned tag, int sender) {
    return cp.buf[q] + kEpCountsOff + (((size_t)(tag & 1u) * kEpMaxRanks + sender) * cp.E) * 8;
}

// Threads [0, nthreads) of the caller write counts[0..E) into rank `peer`'s slot.  The words
// go out as atomic exchanges (result unused): an atomic is performed at the destination at
// once, where a plain store may stay in this GPU until the kernel ends, holding back a kernel
// that goes on (or waits for the peer's row); a system-scope fence after the stores would
// flush them too, but it stalls the writing CTA for the NVLink round trip.
__device__ __forceinline__ bool count_push_failed(const CountPush& cp) {
    return ep_ld_volatile(reinterpret_cast<const unsigned*>(cp.buf[cp.rank] + kEpErr)) != 0u;
}

// A group whose error word is set sends nothing (its peers' waits give up in turn).
__device__ __forceinline__ void count_push_send(const CountPush& cp, const int* counts, int peer,
                                                unsigned tag, int tid, int nthreads) {
    if (count_push_failed(cp)) return;
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(count_slot(cp, peer, tag, cp.rank));
    for (int e = tid; e < cp.E; e += nthreads)
        ep_exch_relaxed_sys_u64(dst + e, ((unsigned long long)tag << 32) | (unsigned)counts[e]);
}

// Whole CTA: wait for every rank's row of this call in this rank's buffer and write
// gathered (-1 and the error word on a wait that gave up, -1 alone when the group had already
// failed); thread 0 then advances the epoch.
// Every thread's polls share one budget: once any wait has given up the others stop too.
__device__ inline void count_push_gather(const CountPush& cp, unsigned tag) {
    __shared__ volatile int lost;
    __shared__ int failed;
    if (threadIdx.x == 0) {
        lost = 0;
        failed = count_push_failed(cp);
    }
    __syncthreads();
    const int n = cp.world * cp.E;
    if (failed) {   // a group whose error word is set: gathered = -1, nothing else
        for (int i = threadIdx.x; i < n; i += blockDim.x) cp.gathered[i] = -1;
        return;
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int q = i / cp.E, e = i - q * cp.E;
        const char* p = count_slot(cp, cp.rank, tag, q) + (size_t)e * 8;
        unsigned long long v = ep_ld_relaxed_sys_u64(p);
        long long it = 0;
        while ((unsigned)(v >> 32) != tag && it < cp.spin && !lost) {
            __nanosleep(64);
            v = ep_ld_relaxed_sys_u64(p);
            ++it;
        }
        if ((unsigned)(v >> 32) == tag) {
            cp.gathered[i] = (int32_t)(unsigned)v;
        } else {
            cp.gathered[i] = -1;
            lost = 1;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (lost) atomicCAS(reinterpret_cast<unsigned*>(cp.buf[cp.rank] + kEpErr), 0u, (unsigned)KB_WS_TIMEOUT);
        *reinterpret_cast<volatile unsigned*>(cp.buf[cp.rank] + kEpCountEpoch) = tag;
    }
}

// Host: the CountPush of a group (declared in ep_peer.cu).  Returns KB_OK or a KB_ERR_*.
int make_count_push(const kb_ep_group_t* g, int32_t* gathered, CountPush* cp);

}  // namespace kb
