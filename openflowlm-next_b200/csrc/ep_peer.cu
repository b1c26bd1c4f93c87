// Expert parallel over peer memory: the exchange kernels of fm_ep_peer_layer.
//
// Each rank's symmetric buffer (identical layout on every rank, EpSym) holds its receive side: the
// count mailbox [G][E], the received rows grouped by expert (+ its own tokens for the shared expert),
// one metadata word per received row (source rank << 24 | the row's position in the source's sorted
// order), the y rows the expert ranks return, and three arrays of monotonic flags (counts posted,
// rows arrived, y rows returned), one slot per source rank. A call's epoch is the local call count;
// a rank publishes a flag by a system-scope release store of the epoch after a system-scope fence
// behind its data stores, and waits with system-scope acquire loads until the flag reaches the epoch.
//
// Every wait is bounded by the group's timeout (globaltimer) and an iteration cap; a wait that gives
// up sets the status word err[1] = FM_ETIMEOUT, and every later step of the call then skips its stores
// to peers and its own signals, so the other ranks time out too instead of waiting for good. A peer's
// buffer is never read: data only moves by stores into the owner's buffer, and the owner reads it
// locally (the tensor-memory GEMM's TMA loads included).
#include "common.cuh"
#include "kernels.cuh"

namespace fm {

__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits until flags[s] >= epoch for every s < G (thread s of the calling warp watches flag s; G <= 32).
// Returns false, after setting err[1] = FM_ETIMEOUT, when the bound runs out or err[1] was already set.
__device__ bool wait_flags(const int* flags, int G, int epoch, int* err, long long timeout_ns) {
    const int lane = threadIdx.x & 31;
    const uint64_t t0 = globaltimer_ns();
    bool ok = true;
    if (lane < G) {
        for (long long it = 0;; ++it) {
            if (ld_acquire_sys(flags + lane) >= epoch) break;
            if (*reinterpret_cast<volatile int*>(err + 1) != 0 || it > (1ll << 26) ||
                (long long)(globaltimer_ns() - t0) > timeout_ns) {
                ok = false;
                break;
            }
            __nanosleep(256);
        }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && lane == 0) atomicCAS(err + 1, 0, FM_ETIMEOUT);
    return ok;
}

// One block: this call's epoch = ++state[0]; counts[E] -> every rank's mailbox row `rank`; then the
// counts-posted flag of this rank on every rank.
__global__ void __launch_bounds__(256) ep_post_counts_kernel(EpPeerArgs a, const int* __restrict__ counts) {
    __shared__ int s_epoch;
    if (threadIdx.x == 0) {
        s_epoch = a.state[0] + 1;
        a.state[0] = s_epoch;
    }
    __syncthreads();
    const bool live = *reinterpret_cast<volatile int*>(a.err + 1) == 0;
    if (live)
        for (int i = threadIdx.x; i < a.G * a.E; i += blockDim.x) {
            const int g = i / a.E, e = i - g * a.E;
            reinterpret_cast<int*>(a.sym[g] + a.off_cnt)[a.rank * a.E + e] = counts[e];
        }
    __threadfence_system();
    __syncthreads();
    if (live && threadIdx.x < a.G)
        st_release_sys(reinterpret_cast<int*>(a.sym[threadIdx.x] + a.off_flags) + 0 * kMaxRanksPad + a.rank, s_epoch);
}

// One block of 1024 threads (E <= 1024): waits for every rank's counts, then
//   send_base[e] = first row, in the owner d = e / El's receive buffer, of this rank's rows for e
//                = (rows of d's experts below e, all sources) + (rows for e from sources below us);
//   seg[j]       = (j, first row, rows) of local expert j in our receive buffer.
// On a timeout every segment is empty, so the GEMMs do nothing.
__global__ void __launch_bounds__(1024) ep_plan_peer_kernel(EpPeerArgs a, int* __restrict__ send_base,
                                                            int* __restrict__ seg) {
    __shared__ int sh[32];
    __shared__ int s_ok;
    const int epoch = a.state[0];
    const int* flags = reinterpret_cast<const int*>(a.sym[a.rank] + a.off_flags) + 0 * kMaxRanksPad;
    if (threadIdx.x < 32) {
        const bool ok = wait_flags(flags, a.G, epoch, a.err, a.timeout_ns);
        if (threadIdx.x == 0) s_ok = ok;
    }
    __syncthreads();
    const int* box = reinterpret_cast<const int*>(a.sym[a.rank] + a.off_cnt);
    const int e = threadIdx.x;
    int tot = 0, pre = 0;
    if (e < a.E && s_ok)
        for (int s = 0; s < a.G; ++s) {
            const int c = box[s * a.E + e];
            tot += c;
            if (s < a.rank) pre += c;
        }
    int all = 0;
    const int ex = block_exclusive_scan(e < a.E ? tot : 0, sh, &all);
    // exclusive scan value at the first expert of e's owner: broadcast through shared memory
    __shared__ int range_start[kMaxRanks];
    if (e < a.E && e % a.El == 0) range_start[e / a.El] = ex;
    __syncthreads();
    if (e < a.E) {
        const int d = e / a.El;
        send_base[e] = ex - range_start[d] + pre;
        if (d == a.rank) {
            const int j = e - a.rank * a.El;
            seg[3 * j] = j;
            seg[3 * j + 1] = ex - range_start[d];
            seg[3 * j + 2] = s_ok ? tot : 0;
        }
    }
}

// Rows -> owners. Warp per sorted row p: pair q = pair[p], token q / k, expert idx[q], owner
// d = expert / El, destination row send_base[e] + (p - offsets[e]) of d's receive buffer (a peer store
// of H bf16, 16 bytes per lane) and its metadata word. After the sorted rows, the walk copies this rank's
// own t_real tokens to its receive buffer's shared-expert rows. The last block to finish publishes the
// rows-arrived flag on every rank (after each block's system-scope fence).
__global__ void __launch_bounds__(256) ep_scatter_rows_kernel(EpPeerArgs a, const uint16_t* __restrict__ xb,
                                                              const int* __restrict__ pair,
                                                              const int32_t* __restrict__ idx,
                                                              const int* __restrict__ offsets,
                                                              const int* __restrict__ send_base, int P, int t_real) {
    const int lane = threadIdx.x & 31;
    const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
    const bool live = *reinterpret_cast<volatile int*>(a.err + 1) == 0;
    // The sorted rows for owner d are the contiguous range [offsets[d El], offsets[(d + 1) El]). The
    // walk interleaves the owners (slot i -> owner i % G, its (i / G)-th row), so that at any moment
    // the stores spread over every peer's links instead of draining one owner after another.
    __shared__ int dstart[kMaxRanks + 1];
    __shared__ int maxlen;
    if (threadIdx.x <= a.G) dstart[threadIdx.x] = offsets[min((int)threadIdx.x * a.El, a.E)];
    __syncthreads();
    if (threadIdx.x == 0) {
        int m = 0;
        for (int d = 0; d < a.G; ++d) m = max(m, dstart[d + 1] - dstart[d]);
        maxlen = m;
    }
    __syncthreads();
    const int nslots = a.G * maxlen;
    if (live) {
        for (int i = wid; i < nslots + t_real; i += nw) {
            const uint4* src;
            uint4* dst;
            if (i < nslots) {
                const int d0 = i % a.G, j = i / a.G;
                if (j >= dstart[d0 + 1] - dstart[d0]) continue;
                const int r = dstart[d0] + j;
                const int q = pair[r];
                const int e = idx[q];
                const int d = e / a.El;
                const int row = send_base[e] + (r - offsets[e]);
                src = reinterpret_cast<const uint4*>(xb + (size_t)(q / a.k) * a.H);
                dst = reinterpret_cast<uint4*>(a.sym[d] + a.off_x + (size_t)row * a.H * 2);
                if (lane == 0) reinterpret_cast<int*>(a.sym[d] + a.off_meta)[row] = (a.rank << 24) | r;
            } else {
                const int t = i - nslots;
                src = reinterpret_cast<const uint4*>(xb + (size_t)t * a.H);
                dst = reinterpret_cast<uint4*>(a.sym[a.rank] + a.off_x + (size_t)(a.r_cap + t) * a.H * 2);
            }
            warp_copy_row(dst, src, a.H / 8, lane);
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int done = atomicAdd(a.state + 1, 1);
        if (done == gridDim.x - 1) {
            a.state[1] = 0;
            __threadfence_system();
            if (*reinterpret_cast<volatile int*>(a.err + 1) == 0) {
                const int epoch = a.state[0];
                for (int g = 0; g < a.G; ++g)
                    st_release_sys(reinterpret_cast<int*>(a.sym[g] + a.off_flags) + 1 * kMaxRanksPad + a.rank, epoch);
            }
        }
    }
}

// One warp: wait for flag array `which` (1 rows arrived, 2 y rows returned) from every rank.
__global__ void ep_wait_kernel(EpPeerArgs a, int which) {
    const int* flags = reinterpret_cast<const int*>(a.sym[a.rank] + a.off_flags) + which * kMaxRanksPad;
    wait_flags(flags, a.G, a.state[0], a.err, a.timeout_ns);
}

// One warp: publish flag array `which` of this rank on every rank (after the kernels before it on the
// stream, whose peer stores were fenced at system scope by their own threads).
__global__ void ep_signal_kernel(EpPeerArgs a, int which) {
    __threadfence_system();
    if (*reinterpret_cast<volatile int*>(a.err + 1) != 0) return;
    const int g = threadIdx.x;
    if (g < a.G) st_release_sys(reinterpret_cast<int*>(a.sym[g] + a.off_flags) + which * kMaxRanksPad + a.rank, a.state[0]);
}

int launch_ep_post_counts(const EpPeerArgs& a, const int* counts, cudaStream_t st) {
    ep_post_counts_kernel<<<1, 256, 0, st>>>(a, counts);
    FM_LAUNCH_CHECK("ep_post_counts");
    return FM_OK;
}

int launch_ep_plan_peer(const EpPeerArgs& a, int* send_base, int* seg, cudaStream_t st) {
    ep_plan_peer_kernel<<<1, 1024, 0, st>>>(a, send_base, seg);
    FM_LAUNCH_CHECK("ep_plan_peer");
    return FM_OK;
}

int launch_ep_scatter_rows(const EpPeerArgs& a, const uint16_t* xb, const int* pair, const int32_t* idx,
                           const int* offsets, const int* send_base, int P, int t_real, int sms, cudaStream_t st) {
    const int rows = P + t_real;
    int grid = (rows + 7) / 8;
    if (grid > 4 * sms) grid = 4 * sms;
    if (grid < 1) grid = 1;
    ep_scatter_rows_kernel<<<grid, 256, 0, st>>>(a, xb, pair, idx, offsets, send_base, P, t_real);
    FM_LAUNCH_CHECK("ep_scatter_rows");
    return FM_OK;
}

int launch_ep_wait(const EpPeerArgs& a, int which, cudaStream_t st) {
    ep_wait_kernel<<<1, 32, 0, st>>>(a, which);
    FM_LAUNCH_CHECK("ep_wait");
    return FM_OK;
}

int launch_ep_signal(const EpPeerArgs& a, int which, cudaStream_t st) {
    ep_signal_kernel<<<1, 32, 0, st>>>(a, which);
    FM_LAUNCH_CHECK("ep_signal");
    return FM_OK;
}

}  // namespace fm
