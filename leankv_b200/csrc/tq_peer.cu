// tq_peer.cu — split-sequence merge of decode-attention partials over peer memory.
//
// The multi-GPU split-KV decode leaves each rank with a packed partial
// [o (n_rows x D) | lse (n_rows)] for its token range; the merged output is the
// log-sum-exp combination of all ranks' partials.  Instead of a collective
// (all_gather) followed by a merge kernel, one kernel per rank does both:
//
//   push   each CTA stores its slice of the local partial into slot (step parity,
//          rank) of every rank's exchange buffer, through the peer mappings
//          opened from CUDA IPC handles (plain stores over NVLink), then a
//          system-scope fence and one 64-bit atomic increment of every rank's
//          arrival counter;
//   wait   one thread per CTA polls its own counter (acquire, system scope)
//          until it reaches step * world * ctas, bounded; a wait that runs out
//          records TQ_ERROR_TIMEOUT in the buffer's status word;
//   merge  rows in rank order, with the arithmetic of lse_combine_kernel, reading
//          the slots through L2 only (ld.global.cg), so the result equals the
//          all_gather + merge path bit for bit.
//
// The counters never reset: step s of an exchange expects s * world * ctas
// arrivals.  A wait is bounded by the exchange's wait limit (%globaltimer,
// 2 s unless the creator chose another); after a wait runs out the exchange
// stays unusable, and recovery is close() plus a new exchange on every rank.
// The grid never exceeds the SM count, so all its CTAs are resident and a
// waiting CTA cannot keep one that still has to push from running.  Slots alternate
// between two buffers by step parity: a rank stores
// step s + 2 into a slot only after its own step s + 1 completed, which needed
// every rank's step s + 1 stores, which every rank issues only after its
// step s merge finished reading that slot.
//
// Buffer of one rank (cudaMalloc, exported with cudaIpcGetMemHandle):
//   [0, 8) arrival counter | [64, 68) status | 256: slots [2][world][slot_floats]
#include <cmath>
#include <cstdint>
#include <cstring>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "leankv_tq.h"
#include "tq_attn.h"
#include "tq_capi_internal.h"
#include "tq_merge.cuh"

namespace {

constexpr int PX_THREADS = 256;
constexpr int PX_ROWS_PER_CTA = PX_THREADS / 32;       // one warp per row in the merge
constexpr int PX_MAX_CTAS = 128;                       // <= SMs: every CTA of the grid is resident
constexpr size_t PX_HEAD = 256;
constexpr size_t PX_STATUS = 64;
constexpr uint32_t PX_DEFAULT_WAIT_MS = 2000;          // bound of the arrival wait when the creator passes 0

struct PeerBases {
    uint8_t* base[TQ_PEER_MAX_WORLD];
};

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// PUSH: store this rank's partial `part` and count every CTA (tq_peer_exchange_merge).  Without it
// the partials were stored and counted by the decode-attention kernel itself
// (tq_peer_exchange_attention): this kernel only waits for the target and merges.
template <typename OT, bool PUSH>
__global__ void __launch_bounds__(PX_THREADS) peer_merge_kernel(const float* __restrict__ part, const PeerBases peers,
                                                                int world, int rank, int64_t n_rows, int D,
                                                                int64_t slot_floats, int par, uint64_t target,
                                                                uint64_t wait_ns, OT* __restrict__ out,
                                                                float* __restrict__ lse_out, int vec) {
    __shared__ int s_ok;
    if (PUSH) {
    // ---- push: this CTA's slice [c0, c1) of the packed partial into every rank's slot ----
    const int64_t F = n_rows * (int64_t)(D + 1);
    const int64_t per = ((F + gridDim.x - 1) / gridDim.x + 3) & ~int64_t(3);   // multiple of 4 floats
    const int64_t c0 = per * blockIdx.x < F ? per * blockIdx.x : F;
    const int64_t c1 = c0 + per < F ? c0 + per : F;
    const int64_t slot_off = ((int64_t)par * world + rank) * slot_floats;
    for (int t = 0; t < world; ++t) {
        float* dst = reinterpret_cast<float*>(peers.base[t] + PX_HEAD) + slot_off;
        int64_t s = c0;
        if (vec) {
            const int64_t v1 = c1 & ~int64_t(3);   // c0 is a multiple of 4; only the last slice has a tail
            for (int64_t c = c0 + 4 * threadIdx.x; c < v1; c += 4 * PX_THREADS)
                *reinterpret_cast<float4*>(dst + c) = __ldg(reinterpret_cast<const float4*>(part + c));
            s = v1;
        }
        for (int64_t c = s + threadIdx.x; c < c1; c += PX_THREADS) dst[c] = part[c];
    }
    __threadfence_system();   // this thread's stores reach every rank before the counts below
    __syncthreads();
    if (threadIdx.x == 0)
        for (int t = 0; t < world; ++t)
            atomicAdd_system(reinterpret_cast<unsigned long long*>(peers.base[t]), 1ull);
    }
    if (threadIdx.x == 0) {
        // ---- wait for every count of every rank (bounded) ----
        const uint64_t* cnt = reinterpret_cast<const uint64_t*>(peers.base[rank]);
        const uint64_t t0 = global_ns();
        while (ld_acquire_sys(cnt) < target && global_ns() - t0 < wait_ns) __nanosleep(64);
        s_ok = ld_acquire_sys(cnt) >= target;
        if (!s_ok) atomicExch(reinterpret_cast<int*>(peers.base[rank] + PX_STATUS), (int)TQ_ERROR_TIMEOUT);
    }
    __syncthreads();
    if (!s_ok) return;

    // ---- merge: one warp per row, ranks in order (merge_row, as lse_combine_kernel) ----
    const float* slots = reinterpret_cast<const float*>(peers.base[rank] + PX_HEAD) + (int64_t)par * world * slot_floats;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t i = (int64_t)blockIdx.x * PX_ROWS_PER_CTA + warp; i < n_rows; i += (int64_t)gridDim.x * PX_ROWS_PER_CTA)
        tq::merge_row<OT>(slots, slot_floats, slots + n_rows * D, slot_floats, world, i, D, out, lse_out, lane);
}

}  // namespace

struct tq_peer_exchange {
    int world = 0, rank = 0, dev = 0, ctas = 0, D = 0;
    int64_t n_rows = 0, slot_floats = 0;
    uint64_t wait_ns = 0;
    uint64_t step = 0;
    uint64_t expected = 0;   // arrivals counted into this rank's counter by the end of the last step
    bool connected = false;
    uint8_t* local = nullptr;
    uint8_t* peer[TQ_PEER_MAX_WORLD] = {};
    bool opened[TQ_PEER_MAX_WORLD] = {};
};

using tq::cuda_status;
using tq::set_error;

static tq_status px_device(const tq_peer_exchange* ex) {
    int dev = -1;
    tq_status s = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (s) return s;
    if (dev != ex->dev)
        return set_error(TQ_ERROR_INVALID_VALUE, "exchange created on device %d, called on device %d", ex->dev, dev);
    return TQ_SUCCESS;
}

extern "C" tq_status tq_peer_exchange_create(int world, int rank, int64_t n_rows, int head_dim, uint32_t wait_ms,
                                             tq_peer_exchange** ex, void* handle_out) {
    if (!ex || !handle_out) return set_error(TQ_ERROR_INVALID_VALUE, "null argument");
    *ex = nullptr;
    if (world < 1 || world > TQ_PEER_MAX_WORLD) return set_error(TQ_ERROR_INVALID_VALUE, "world %d outside [1, 64]", world);
    if (rank < 0 || rank >= world) return set_error(TQ_ERROR_INVALID_VALUE, "rank %d outside [0, world)", rank);
    if (n_rows <= 0 || head_dim <= 0 || head_dim > 4096)
        return set_error(TQ_ERROR_INVALID_VALUE, "bad n_rows / head_dim");
    static_assert(sizeof(cudaIpcMemHandle_t) == TQ_PEER_HANDLE_BYTES, "IPC handle size");
    tq_peer_exchange* e = new tq_peer_exchange();
    e->world = world;
    e->rank = rank;
    e->n_rows = n_rows;
    e->D = head_dim;
    e->slot_floats = (n_rows * (int64_t)(head_dim + 1) + 63) / 64 * 64;   // slots start 256-byte aligned
    e->wait_ns = (uint64_t)(wait_ms ? wait_ms : PX_DEFAULT_WAIT_MS) * 1000000ull;
    tq_status s = cuda_status(cudaGetDevice(&e->dev), "cudaGetDevice");
    int sms = 0;
    if (!s) s = cuda_status(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, e->dev), "SM count");
    int64_t ctas = (n_rows + PX_ROWS_PER_CTA - 1) / PX_ROWS_PER_CTA;
    if (ctas > PX_MAX_CTAS) ctas = PX_MAX_CTAS;
    if (sms > 0 && ctas > sms) ctas = sms;   // every CTA of the grid resident: no waiting CTA starves a pusher
    e->ctas = (int)ctas;
    const size_t bytes = PX_HEAD + (size_t)2 * world * e->slot_floats * sizeof(float);
    if (!s) s = cuda_status(cudaMalloc(&e->local, bytes), "cudaMalloc(exchange buffer)");
    if (!s) s = cuda_status(cudaMemset(e->local, 0, PX_HEAD), "cudaMemset(exchange counters)");
    cudaIpcMemHandle_t h;
    if (!s) s = cuda_status(cudaIpcGetMemHandle(&h, e->local), "cudaIpcGetMemHandle");
    if (s) {
        if (e->local) cudaFree(e->local);
        delete e;
        return s;
    }
    std::memcpy(handle_out, &h, sizeof(h));
    *ex = e;
    return TQ_SUCCESS;
}

extern "C" tq_status tq_peer_exchange_connect(tq_peer_exchange* ex, const void* handles) {
    if (!ex || !handles) return set_error(TQ_ERROR_INVALID_VALUE, "null argument");
    if (ex->connected) return set_error(TQ_ERROR_INVALID_VALUE, "exchange already connected");
    tq_status s = px_device(ex);
    if (s) return s;
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (int t = 0; t < ex->world; ++t) {
        if (t == ex->rank) {
            ex->peer[t] = ex->local;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + (size_t)t * TQ_PEER_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        s = cuda_status(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
        if (s) {
            tq_peer_exchange_disconnect(ex);
            return s;
        }
        ex->peer[t] = static_cast<uint8_t*>(p);
        ex->opened[t] = true;
    }
    ex->connected = true;
    return TQ_SUCCESS;
}

template <bool PUSH>
static tq_status launch_merge(tq_peer_exchange* ex, const float* part, void* out, tq_dtype out_dtype, float* lse_out,
                              uint64_t target, cudaStream_t st) {
    PeerBases pb;
    for (int t = 0; t < TQ_PEER_MAX_WORLD; ++t) pb.base[t] = t < ex->world ? ex->peer[t] : nullptr;
    const uint64_t step = ex->step + 1;
    const int par = (int)(step & 1);
    const int vec = part && (((uintptr_t)part) & 15) == 0;
    switch (out_dtype) {
        case TQ_DTYPE_F32:
            peer_merge_kernel<float, PUSH><<<ex->ctas, PX_THREADS, 0, st>>>(
                part, pb, ex->world, ex->rank, ex->n_rows, ex->D, ex->slot_floats, par, target, ex->wait_ns,
                (float*)out, lse_out, vec);
            break;
        case TQ_DTYPE_F16:
            peer_merge_kernel<__half, PUSH><<<ex->ctas, PX_THREADS, 0, st>>>(
                part, pb, ex->world, ex->rank, ex->n_rows, ex->D, ex->slot_floats, par, target, ex->wait_ns,
                (__half*)out, lse_out, vec);
            break;
        default:
            peer_merge_kernel<__nv_bfloat16, PUSH><<<ex->ctas, PX_THREADS, 0, st>>>(
                part, pb, ex->world, ex->rank, ex->n_rows, ex->D, ex->slot_floats, par, target, ex->wait_ns,
                (__nv_bfloat16*)out, lse_out, vec);
            break;
    }
    const tq_status s = cuda_status(cudaGetLastError(), "peer merge launch");
    if (!s) ex->step = step;
    return s;
}

extern "C" tq_status tq_peer_exchange_attention(tq_peer_exchange* ex, const tq_decode_attention_args* a, void* out,
                                                tq_dtype out_dtype, float* lse_out, void* stream) {
    if (!ex || !a || !out) return set_error(TQ_ERROR_INVALID_VALUE, "null argument");
    if (!ex->connected) return set_error(TQ_ERROR_INVALID_VALUE, "exchange not connected");
    if (!tq::dtype_ok(out_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "bad output dtype");
    if (((uintptr_t)out) % tq::dtype_bytes(out_dtype)) return set_error(TQ_ERROR_MISALIGNED, "out not aligned");
    tq_status s = px_device(ex);
    if (s) return s;
    tq::AttnRun r;
    tq::AttnPlan p;
    if ((s = tq::attn_check(a, &r, &p))) return s;
    if ((int64_t)r.B * r.Hq != ex->n_rows || r.D != ex->D)
        return set_error(TQ_ERROR_INVALID_VALUE, "batch * n_q_heads = %lld and head_dim %d do not match the exchange "
                         "(%lld rows of %d)", (long long)r.B * r.Hq, r.D, (long long)ex->n_rows, ex->D);
    const size_t need = tq::attn_workspace_bytes(r.B, r.Hkv, r.D, p);
    if (!a->workspace || a->workspace_bytes < need)
        return set_error(TQ_ERROR_INVALID_VALUE, "workspace of %zu bytes needed", need);
    if (((uintptr_t)a->workspace) & 255) return set_error(TQ_ERROR_MISALIGNED, "workspace must be 256-byte aligned");
    if (r.D % 4) return set_error(TQ_ERROR_UNSUPPORTED, "head_dim must be a multiple of 4");
    // the decode kernel stores its (o, lse) rows into step (ex->step + 1)'s slot of every rank and
    // counts each (sequence, KV head) pair there; the merge kernel waits for all ranks' pairs
    r.peer.world = ex->world;
    r.peer.rank = ex->rank;
    r.peer.par = (int)((ex->step + 1) & 1);
    r.peer.slot_floats = ex->slot_floats;
    r.peer.n_rows = ex->n_rows;
    for (int t = 0; t < ex->world; ++t) r.peer.base[t] = ex->peer[t];
    const cudaStream_t st = (cudaStream_t)stream;
    s = cuda_status(tq::launch_decode_attention(r, p, a->workspace, st), "decode attention launch");
    if (s) return s;   // nothing was counted: the step and the targets stay where the peers expect them
    const uint64_t target = ex->expected + (uint64_t)ex->world * (uint64_t)r.B * (uint64_t)r.Hkv;
    s = launch_merge<false>(ex, nullptr, out, out_dtype, lse_out, target, st);
    if (!s) ex->expected = target;
    return s;
}

extern "C" tq_status tq_peer_exchange_merge(tq_peer_exchange* ex, const float* part, void* out, tq_dtype out_dtype,
                                            float* lse_out, void* stream) {
    if (!ex || !part || !out) return set_error(TQ_ERROR_INVALID_VALUE, "null argument");
    if (!ex->connected) return set_error(TQ_ERROR_INVALID_VALUE, "exchange not connected");
    if (!tq::dtype_ok(out_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "bad output dtype");
    if (((uintptr_t)part) & 3) return set_error(TQ_ERROR_MISALIGNED, "part not aligned to 4 bytes");
    if (((uintptr_t)out) % tq::dtype_bytes(out_dtype)) return set_error(TQ_ERROR_MISALIGNED, "out not aligned");
    tq_status s = px_device(ex);
    if (s) return s;
    const uint64_t target = ex->expected + (uint64_t)ex->world * (uint64_t)ex->ctas;
    s = launch_merge<true>(ex, part, out, out_dtype, lse_out, target, (cudaStream_t)stream);
    if (!s) ex->expected = target;   // a launch that failed leaves the counts where the peers expect them
    return s;
}

extern "C" tq_status tq_peer_exchange_status(tq_peer_exchange* ex, void* stream) {
    if (!ex) return set_error(TQ_ERROR_INVALID_VALUE, "null argument");
    tq_status s = px_device(ex);
    if (s) return s;
    s = cuda_status(cudaStreamSynchronize((cudaStream_t)stream), "cudaStreamSynchronize");
    if (s) return s;
    int v = 0;
    s = cuda_status(cudaMemcpy(&v, ex->local + PX_STATUS, sizeof(int), cudaMemcpyDeviceToHost), "status read");
    if (s) return s;
    if (v == TQ_ERROR_TIMEOUT) return set_error(TQ_ERROR_TIMEOUT, "a peer exchange wait ran out");
    if (v != 0) return set_error((tq_status)v, "peer exchange kernel status %d", v);
    return TQ_SUCCESS;
}

extern "C" tq_status tq_peer_exchange_disconnect(tq_peer_exchange* ex) {
    if (!ex) return set_error(TQ_ERROR_INVALID_VALUE, "null argument");
    tq_status first = TQ_SUCCESS;
    for (int t = 0; t < ex->world; ++t) {
        if (ex->opened[t]) {
            const tq_status s = cuda_status(cudaIpcCloseMemHandle(ex->peer[t]), "cudaIpcCloseMemHandle");
            if (s && !first) first = s;
            ex->opened[t] = false;
        }
        ex->peer[t] = nullptr;
    }
    ex->connected = false;
    return first;
}

extern "C" tq_status tq_peer_exchange_destroy(tq_peer_exchange* ex) {
    if (!ex) return TQ_SUCCESS;
    tq_status s = TQ_SUCCESS;
    if (ex->connected) s = tq_peer_exchange_disconnect(ex);
    if (ex->local) {
        const tq_status f = cuda_status(cudaFree(ex->local), "cudaFree(exchange buffer)");
        if (!s) s = f;
    }
    delete ex;
    return s;
}
