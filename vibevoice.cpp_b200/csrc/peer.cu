// peer.cu -- the exchanges of a partitioned decode step over NVLink peer
// memory, each fused with the computation that consumes it (sm_100a).
//
// A partitioned context (vvq2_partition) splits a layer's attention by KV
// head group and sequence part and its FFN by intermediate features; every
// layer then needs (1) the attention output of all ranks' heads, merged over
// the sequence parts, as the O-projection input, and (2) the sum of all
// ranks' partial down projections, added to the residual stream
// (src/vibevoice_asr.cpp:554-652 runs this stack; src/qwen2.cpp:327-355 the
// layer).  For the one or two token rows of a decode step these messages
// are a few KB: a library collective per exchange costs more in launch and
// protocol latency than the data takes to cross NVLink.  Here each rank owns
// one exchange buffer, mapped into every other rank's address space (CUDA
// IPC), and one single-CTA kernel per exchange
//   - stores this rank's block into slot [parity][rank] of every rank's
//     buffer (plain peer stores),
//   - publishes it with a system-scope release store of the call's epoch
//     into flag [rank] of every rank's buffer,
//   - waits (bounded) until every rank's flag in its own buffer shows the
//     epoch, and
//   - computes its output from the slots: the rank-order sum plus the
//     residual add, or the heads of all groups with the two sequence parts
//     merged by log-sum-exp.
// The epoch comes from a device counter each kernel advances, so every
// rank, running the same exchanges in the same order, agrees on it without
// the host.  Slots alternate by epoch parity: a rank cannot start exchange
// e + 2 before every rank has finished reading exchange e (it would have
// had to see their e + 1 flags, which they raise only after reading e).
// No TMA and no bulk copy touches peer memory; a wait that runs out sets
// the context's error word and the kernel returns.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace vvq2 {

namespace {

constexpr int PX_THREADS = 1024;
constexpr unsigned long long PX_WAIT_NS = 1000000000ull;   // a wait for a peer gives up after 1 s
constexpr uint32_t PX_POLLS = 1u << 26;                     // and after this many polls in any case

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint8_t* slot(const PeerArgs& p, int owner, int parity, int sender) {
    return p.base[owner] + PEER_HDR + ((size_t)parity * PEER_MAX + sender) * p.slot_bytes;
}

__device__ __forceinline__ void push(const PeerArgs& p, int par, const void* src, int bytes, int off) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x) {
        const uint4 v = s4[i];
        for (int r = 0; r < p.world; ++r) reinterpret_cast<uint4*>(slot(p, r, par, p.rank) + off)[i] = v;
    }
}

// Push this rank's block -- bytes0 from src0, then bytes1 from src1 at the
// next 16-byte boundary (both multiples of 16, src1 may be null) -- into
// slot [parity][rank] of every rank, publish, and wait for every rank's
// block of this epoch.  Returns the epoch's parity, or -1 after a wait ran
// out (error word set).  All threads of the CTA call it.
__device__ int exchange(const PeerArgs& p, const void* src0, int bytes0, const void* src1, int bytes1,
                        unsigned int* s_epoch, int* s_ok) {
    if (threadIdx.x == 0) {
        *s_epoch = *p.epoch + 1;
        *s_ok = 1;
    }
    __syncthreads();
    const unsigned int e = *s_epoch;
    const int par = e & 1;
    push(p, par, src0, bytes0, 0);
    if (src1) push(p, par, src1, bytes1, bytes0);
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();   // every thread's peer stores before the flags
        for (int r = 0; r < p.world; ++r)
            st_release_sys(reinterpret_cast<unsigned int*>(p.base[r]) + p.rank, e);
    }
    if (threadIdx.x < p.world) {
        const unsigned int* f = reinterpret_cast<const unsigned int*>(p.base[p.rank]) + threadIdx.x;
        uint32_t it = 0;
        const unsigned long long t0 = gtimer();
        while (ld_acquire_sys(f) != e) {
            if (++it > PX_POLLS || ((it & 255) == 0 && gtimer() - t0 > PX_WAIT_NS)) {
                atomicExch(s_ok, 0);
                if (p.err) atomicExch(p.err, 6);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *p.epoch = e;
    return *s_ok ? par : -1;
}

// x[i] += sum over ranks r (in rank order) of part_r[i], i < n
__global__ void __launch_bounds__(PX_THREADS) k_peer_reduce_add(PeerArgs p, const float* part, int n, float* x) {
    __shared__ unsigned int s_epoch;
    __shared__ int s_ok;
    const int par = exchange(p, part, n * 4, nullptr, 0, &s_epoch, &s_ok);
    if (par < 0) return;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = 0.f;
        for (int r = 0; r < p.world; ++r) v = __fadd_rn(v, reinterpret_cast<const float*>(slot(p, p.rank, par, r))[i]);
        x[i] = __fadd_rn(x[i], v);
    }
}

// The attention output of every rank -- block [M][nq_l * hd] f16, then (two
// sequence parts) its log-sum-exps [M][nq_l] -- into out [M][nq * hd] f32:
// head h of row m comes from head group g = h / nq_l, ranks g * seq_parts +
// s; two parts merge as (w0 o0 + w1 o1) / (w0 + w1), w_s = exp(l_s - max),
// rounded to f16 like the output of one part.
__global__ void __launch_bounds__(PX_THREADS) k_peer_attn_gather(PeerArgs p, const __half* o, const float* lse, int M,
                                                                 int nq_l, int hd, int seq_parts, float* out) {
    __shared__ unsigned int s_epoch;
    __shared__ int s_ok;
    const int ob = (M * nq_l * hd * 2 + 15) / 16 * 16;
    const int par = exchange(p, o, ob, seq_parts == 2 ? lse : nullptr, (M * nq_l * 4 + 15) / 16 * 16, &s_epoch, &s_ok);
    if (par < 0) return;
    const int groups = p.world / seq_parts, qw_l = nq_l * hd, qw = groups * qw_l;
    for (int i = threadIdx.x; i < M * qw; i += blockDim.x) {
        const int m = i / qw, c = i % qw, g = c / qw_l, j = c % qw_l;
        const int r0 = g * seq_parts;
        const __half* o0 = reinterpret_cast<const __half*>(slot(p, p.rank, par, r0));
        float v = __half2float(o0[(size_t)m * qw_l + j]);
        if (seq_parts == 2) {
            const __half* o1 = reinterpret_cast<const __half*>(slot(p, p.rank, par, r0 + 1));
            const size_t lo = (size_t)ob / 4 + (size_t)m * nq_l + j / hd;
            const float l0 = reinterpret_cast<const float*>(slot(p, p.rank, par, r0))[lo];
            const float l1 = reinterpret_cast<const float*>(slot(p, p.rank, par, r0 + 1))[lo];
            const float mx = fmaxf(l0, l1);
            float w = 0.f;
            if (mx != -INFINITY) {
                const float w0 = expf(l0 - mx), w1 = expf(l1 - mx);
                w = (w0 * v + w1 * __half2float(o1[(size_t)m * qw_l + j])) / (w0 + w1);
            }
            v = __half2float(__float2half_rn(w));
        }
        out[i] = v;
    }
}

}  // namespace

cudaError_t peer_reduce_add_launch(const PeerArgs& p, const float* part, int n, float* x, cudaStream_t st) {
    if (n % 4 || (size_t)n * 4 > (size_t)p.slot_bytes) return cudaErrorInvalidValue;
    k_peer_reduce_add<<<1, PX_THREADS, 0, st>>>(p, part, n, x);
    note_launch();
    return cudaGetLastError();
}

int peer_attn_block_bytes(int M, int nq_l, int hd, int seq_parts) {
    const int ob = ((M * nq_l * hd * 2) + 15) / 16 * 16;
    return seq_parts == 2 ? ob + (M * nq_l * 4 + 15) / 16 * 16 : ob;
}

cudaError_t peer_attn_gather_launch(const PeerArgs& p, const __half* o, const float* lse, int M, int nq_l, int hd,
                                    int seq_parts, float* out, cudaStream_t st) {
    const int bytes = peer_attn_block_bytes(M, nq_l, hd, seq_parts);
    if (bytes > p.slot_bytes || (seq_parts != 1 && seq_parts != 2) || p.world % seq_parts || (seq_parts == 2 && !lse))
        return cudaErrorInvalidValue;
    k_peer_attn_gather<<<1, PX_THREADS, 0, st>>>(p, o, lse, M, nq_l, hd, seq_parts, out);
    note_launch();
    return cudaGetLastError();
}

}  // namespace vvq2
