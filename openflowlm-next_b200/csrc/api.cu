// The C ABI of libflowmoe.so (declared in include/flowmoe.h): argument checks, the workspace layout
// and the launch sequence of each entry point. No entry point allocates device memory: the caller
// passes the workspace (fm_workspace_size) and every output buffer.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "kernels.cuh"

namespace fm {

static thread_local char g_err[512];
static std::atomic<unsigned long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool pdl_on() {
    static const bool on = [] {
        const char* v = std::getenv("FLOWMOE_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

int device_sm_count() {
    constexpr int kDevs = 64;
    static std::atomic<int> cache[kDevs] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
    if (dev < kDevs) {
        const int c = cache[dev].load(std::memory_order_relaxed);
        if (c > 0) return c;
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev < kDevs) cache[dev].store(n, std::memory_order_relaxed);
    return n;
}

cudaError_t raise_smem_limit(const void* func, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<int, const void*>, int> limit;   // the largest limit set so far
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    int& cur = limit[std::make_pair(dev, func)];
    if (bytes <= cur) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) cur = bytes;
    return e;
}

// Stage profiler: pairs of timing events recorded around each stage while enabled; read back (and
// summed per stage) by fm_profile_read. Events are created when profiling is first enabled.
struct Profiler {
    bool on = false;
    static constexpr int kPairs = 1024;
    cudaEvent_t ev[kPairs][2] = {};
    int stage[kPairs] = {};
    int n = 0;
    int open[kStageCount] = {};   // pair index of the stage's open event, -1 when none
};
static thread_local Profiler g_prof;

// An event record that is a graph node inside a stream capture and a plain record outside it.
static void prof_record(cudaEvent_t ev, cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs == cudaStreamCaptureStatusActive) cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal);
    else cudaEventRecord(ev, st);
}

void prof_begin(int stage, cudaStream_t st) {
    if (!g_prof.on) return;
    if (g_prof.n >= Profiler::kPairs) {   // table full: this stage goes unrecorded
        g_prof.open[stage] = -1;
        return;
    }
    const int i = g_prof.n++;
    g_prof.stage[i] = stage;
    g_prof.open[stage] = i;
    prof_record(g_prof.ev[i][0], st);
}

void prof_end(int stage, cudaStream_t st) {
    if (!g_prof.on) return;
    const int i = g_prof.open[stage];
    if (i >= 0 && i < g_prof.n && g_prof.stage[i] == stage) prof_record(g_prof.ev[i][1], st);
    g_prof.open[stage] = -1;
}

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int cuda_status(cudaError_t e, const char* what) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return FM_ECUDA;
}

// kernels: see kernels.cuh

constexpr int kBN = 64;        // rows per work item the list sizes assume (>= the real items' rows)
constexpr int kBNTc = kTcItemRows;   // rows per expert work item (expert_tc)
constexpr int kFlagTc = 2, kFlagGemv = 3;   // 1 and 4 were retired kernel variants
constexpr int kFlagPath = 0xFF;                // the kernel choice bits of fm_layer.flags
// FM_FIXED_ORDER (include/flowmoe.h): every token's expert terms added in ascending expert order, so a
// call's output is bit-reproducible and does not depend on the other tokens in the call
static bool fixed_order(const fm_layer* L) { return (L->flags & FM_FIXED_ORDER) != 0; }

// The GEMV path up to this many tokens, auto or forced (flags = 3), while T * top_k <= 1024 (the
// single-CTA dispatch). Measured on B200 from 48 to 128 tokens (C30 and C36 layers): 2.2-2.5x faster
// than the tcgen05 path, which needs more rows per expert to amortise its dequantisation.
constexpr int kDecodeMaxT = 128;
constexpr int kGemvMaxT = 128;

static int gemv_max_t(const fm_layer* L) { return (L->flags & kFlagPath) == kFlagGemv ? kGemvMaxT : kDecodeMaxT; }
constexpr int kGemvRowsApi = 8;    // sorted rows per GEMV item (decode.cu)
constexpr int kChunk = 2048;   // dispatch chunk (dispatch.cu)

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// A second stream and fork / join events per device (the shared expert runs beside the dispatch and
// the row exchange). Created on the first call, outside any stream capture.
struct SideStream {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
    // Held while one call enqueues its side work, so that another host thread cannot re-record `fork`
    // between this call's record and the side stream's wait on it. (A later `join` record only makes a
    // waiter wait for more of the side stream's FIFO work, never for less.)
    std::mutex enqueue;
};

static SideStream* side_stream() {
    static SideStream per_dev[64];
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    SideStream& x = per_dev[dev];
    if (!x.s) {
        if (cudaStreamCreateWithFlags(&x.s, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&x.fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&x.join, cudaEventDisableTiming) != cudaSuccess) {
            x.s = nullptr;
            return nullptr;
        }
    }
    return &x;
}


// Creates this device's side stream and its events now (fm_moe_layer_noalloc's first-call set-up), so
// that no later call creates them.
int prepare_side_stream() {
    if (!side_stream()) {
        set_error("could not create the side stream");
        return FM_ECUDA;
    }
    return FM_OK;
}

struct Layout {
    size_t err, xb, logits, counts, offsets, blk_hist, pos, pair, gu_list, dn_list, xperm, hperm, yperm, sgate, idx, w;
    size_t part, done, gu_list_sh, dn_list_sh;
    size_t total;
    int nblk, max_gu, max_dn, P, rows, fmax, max_slots, part_cols, kc_cap;
};

static int validate(const fm_layer* L, int T) {
    if (!L) {
        set_error("null layer");
        return FM_EINVAL_SHAPE;
    }
    const int H = L->hidden, E = L->n_experts, k = L->top_k, F = L->ffn, FS = L->shared_ffn;
    if (H <= 0 || H % kTileRows || E <= 0 || E > 1024 || F <= 0 || F % 64 || FS < 0 || FS % 64 || T < 0) {
        set_error("bad geometry H=%d E=%d F=%d F_s=%d T=%d (H %% 128, F and F_s %% 64 == 0, E <= 1024)", H, E, F, FS, T);
        return FM_EINVAL_SHAPE;
    }
    if (k <= 0 || k > E || k > kMaxTopK) {
        set_error("router_block: topk %d past the expert count %d (or > %d)", k, E, kMaxTopK);
        return FM_EINVAL_SHAPE;
    }
    const int path = L->flags & kFlagPath;
    if ((L->flags & ~(kFlagPath | FM_FIXED_ORDER)) || (path != 0 && path != kFlagTc && path != kFlagGemv)) {
        set_error("flags 0x%x: the kernel choice is 0 (size default), 2 (tcgen05) or 3 (GEMV), plus FM_FIXED_ORDER",
                  L->flags);
        return FM_EINVAL_SHAPE;
    }
    if (L->e_begin < 0 || L->e_local < 0 || L->e_begin + L->e_local > E) {
        set_error("bad local expert range [%d, %d) of %d", L->e_begin, L->e_begin + L->e_local, E);
        return FM_EINVAL_SHAPE;
    }
    return FM_OK;
}

static Layout make_layout(const fm_layer* L, int T) {
    Layout o{};
    const int H = L->hidden, E = L->n_experts, k = L->top_k;
    o.P = T * k;
    o.rows = o.P + T;
    o.fmax = L->ffn > L->shared_ffn ? L->ffn : L->shared_ffn;
    o.nblk = (o.P + kChunk - 1) / kChunk;
    const int G = L->e_local + 1;
    const int rt_routed = o.P / kBN + L->e_local;       // >= sum over routed groups of ceil(cnt / kBN)
    const int rt_shared = (T + kBN - 1) / kBN;
    o.max_gu = rt_routed * (L->ffn / 64) + rt_shared * (L->shared_ffn / 64);
    o.max_dn = (rt_routed + (L->shared_ffn ? rt_shared : 0)) * (H / kTileRows);
    const bool decode = T <= gemv_max_t(L);
    if (decode) {
        // GEMV items: 16-row tiles, up to 4 K chunks each
        const int tt = o.P / kGemvRowsApi + L->e_local + (T + kGemvRowsApi - 1) / kGemvRowsApi;
        const int bands = (L->ffn > L->shared_ffn ? L->ffn : L->shared_ffn) / 64;
        o.max_slots = tt * (bands > H / kTileRows ? bands : H / kTileRows);
        o.kc_cap = gemv_chunk_cap(T);
        if (o.kc_cap * o.max_slots > o.max_gu) o.max_gu = o.kc_cap * o.max_slots;
        if (o.kc_cap * o.max_slots > o.max_dn) o.max_dn = o.kc_cap * o.max_slots;
        o.part_cols = 2 * o.fmax > H ? 2 * o.fmax : H;
    }
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t at = off; off = align256(off + bytes); return at; };
    o.err = take(16);   // first: fm_moe_check reads the counter at the workspace start
    o.xb = take((size_t)T * H * 2);
    o.logits = take(router_scratch_bytes(T, H, E, fixed_order(L)));
    o.counts = take((size_t)G * 4);
    o.offsets = take((size_t)(G + 1) * 4);
    o.blk_hist = take((size_t)o.nblk * L->e_local * 4);
    o.pos = take((size_t)o.P * 4);
    o.pair = take((size_t)o.P * 4);
    o.gu_list = take((size_t)(4 + 4 * o.max_gu) * 4);
    o.dn_list = take((size_t)(4 + 4 * o.max_dn) * 4);
    o.xperm = take((size_t)o.rows * H * 2);
    o.hperm = take((size_t)o.rows * o.fmax * 2);
    // f32 y rows: the GEMV path, and the tcgen05 path's fixed-order combine
    o.yperm = take(decode || fixed_order(L) ? (size_t)o.rows * H * 4 : 0);
    o.sgate = take((size_t)T * 4);
    o.idx = take((size_t)o.P * 4);
    o.w = take((size_t)o.P * 4);
    o.gu_list_sh = take((size_t)(4 + 4 * rt_shared * (L->shared_ffn / 64)) * 4);
    o.dn_list_sh = take((size_t)(4 + 4 * rt_shared * (H / kTileRows)) * 4);
    if (decode) {
        o.part = take(o.kc_cap > 1 ? (size_t)o.kc_cap * o.rows * o.part_cols * 4 : 0);   // K chunks only
        o.done = take((size_t)kGemvWarps * o.max_slots * 4);
    }
    o.total = off;
    return o;
}

template <class T>
static T* at(void* ws, size_t off) { return reinterpret_cast<T*>(static_cast<char*>(ws) + off); }

static int check_ws(const Layout& lo, void* ws, size_t bytes) {
    if (lo.total > 0 && (!ws || bytes < lo.total)) {
        set_error("workspace of %zu B is smaller than the %zu B needed", bytes, lo.total);
        return FM_EWORKSPACE;
    }
    if (reinterpret_cast<uintptr_t>(ws) & 255) {
        set_error("workspace must be 256-byte aligned");
        return FM_EWORKSPACE;
    }
    return FM_OK;
}

// Clears the call's status words (expert ids out of range, device waits that gave up) before its first
// kernel on the tcgen05 path; on the GEMV path the dispatch kernel clears them itself.
static int clear_status(void* ws, const Layout& lo, cudaStream_t st) {
    if (cudaMemsetAsync(at<int>(ws, lo.err), 0, 16, st) != cudaSuccess) return cuda_status(cudaGetLastError(), "memset");
    return FM_OK;
}

static int xm_to_bf16(const fm_layer* L, const void* xm, int dtype, int T, void* ws, const Layout& lo,
                      const uint16_t** xb, cudaStream_t st) {
    if (dtype == FM_BF16) {
        *xb = static_cast<const uint16_t*>(xm);
        return FM_OK;
    }
    if (dtype != FM_F32) {
        set_error("xm dtype %d is neither FM_F32 nor FM_BF16", dtype);
        return FM_EINVAL_SHAPE;
    }
    *xb = at<uint16_t>(ws, lo.xb);
    prof_begin(kStageToBf16, st);
    const int rc = launch_to_bf16(static_cast<const float*>(xm), at<uint16_t>(ws, lo.xb), (long long)T * L->hidden, st);
    prof_end(kStageToBf16, st);
    return rc;
}

enum class Path { Tc, Gemv };

// The GEMV up to kDecodeMaxT tokens (while T * top_k <= 1024, the single-CTA dispatch, and fewer than
// 1024 local experts), the tcgen05 grouped GEMM otherwise; flags force either (the GEMV only within its
// limits).
static Path pick_path(const fm_layer* L, int T) {
    const bool gemv_ok = T <= gemv_max_t(L) && L->e_local < 1024 && T * L->top_k <= 1024;
    switch (L->flags & kFlagPath) {
        case kFlagTc: return Path::Tc;
        default: break;
    }
    return gemv_ok ? Path::Gemv : Path::Tc;
}

static int run_block_gemv(const fm_layer* L, const uint16_t* xb, const float* res, const int32_t* idx, const float* w,
                          const float* sgate, int T, int t_real, float* out, void* ws, const Layout& lo,
                          cudaStream_t st) {
    const int H = L->hidden, k = L->top_k;
    const bool shared_on = L->shared_ffn > 0 && sgate && L->shared_gate_up && L->shared_down && t_real > 0;
    const int P = t_real * k, Pcap = lo.P;
    // the dispatch kernel clears the status words, except in the fixed-order mode, where the caller did
    // before the router (whose tcgen05 kernel may report a timeout)
    prof_begin(kStageDispatch, st);
    int rc = launch_dispatch_small(idx, P, L->e_begin, L->e_local, Pcap, shared_on ? t_real : 0, at<int>(ws, lo.counts),
                                   at<int>(ws, lo.offsets), at<int>(ws, lo.pos), at<int>(ws, lo.pair),
                                   at<int>(ws, lo.gu_list), L->ffn / 64, shared_on ? L->shared_ffn / 64 : 0,
                                   H / kTileK, at<int>(ws, lo.dn_list), H / kTileRows, L->ffn / kTileK,
                                   shared_on ? L->shared_ffn / kTileK : L->ffn / kTileK, lo.kc_cap,
                                   fixed_order(L) ? 0 : 1, fixed_order(L) ? 0 : 1, at<int>(ws, lo.done),
                                   at<int>(ws, lo.err), st);
    if (rc) return rc;
    prof_end(kStageDispatch, st);
    GemvLaunch g{};
    g.max_items = lo.max_gu;
    g.list = at<int>(ws, lo.gu_list);
    g.w_routed = L->gate_up;
    g.w_routed_stride = (size_t)2 * L->ffn * H / 32 * 20;
    g.w_shared = L->shared_gate_up;
    g.shared_group = L->e_local;
    g.K_routed = H;
    g.K_shared = H;
    g.act = xb;
    g.act_ld = H;
    g.pair = at<int>(ws, lo.pair);
    g.k = k;
    g.shared_base = Pcap;
    g.part = at<float>(ws, lo.part);
    g.part_rows = lo.rows;
    g.part_ld = lo.part_cols;
    g.done = at<int>(ws, lo.done);
    g.h_out = at<uint16_t>(ws, lo.hperm);
    g.h_ld = lo.fmax;
    g.F_routed = L->ffn;
    g.F_shared = L->shared_ffn;
    g.dn_list = at<int>(ws, lo.dn_list);
    g.y_out = at<float>(ws, lo.yperm);
    g.y_rows = lo.rows;
    g.H = H;
    g.err = at<int>(ws, lo.err) + 1;
    g.tc_min = fixed_order(L) ? 8 : 1;
    prof_begin(kStageGateUp, st);
    if ((rc = launch_gemv(true, g, st))) return rc;
    prof_end(kStageGateUp, st);
    GemvLaunch d = g;
    d.max_items = lo.max_dn;
    d.list = at<int>(ws, lo.dn_list);
    d.w_routed = L->down;
    d.w_routed_stride = (size_t)H * L->ffn / 32 * 20;
    d.w_shared = L->shared_down;
    d.K_routed = L->ffn;
    d.K_shared = L->shared_ffn;
    d.act = at<uint16_t>(ws, lo.hperm);
    d.act_ld = lo.fmax;
    d.done = nullptr;   // K chunks of the down GEMM add into y
    d.y_out = at<float>(ws, lo.yperm);
    d.H = H;
    prof_begin(kStageDown, st);
    if ((rc = launch_gemv(false, d, st))) return rc;
    prof_end(kStageDown, st);
    prof_begin(kStageCombine, st);
    rc = launch_combine(res, at<float>(ws, lo.yperm), at<int>(ws, lo.pos), idx, w, sgate, shared_on ? 1 : 0, T, t_real,
                        k, H, Pcap, out, st);
    prof_end(kStageCombine, st);
    return rc;
}

// The shared expert as its own pair of tcgen05 launches on the side stream (forked from st at this
// point): gate_up over x rows [0, t_real) straight from xb, h into h_rows, down adding
// sgate * y into out. Leaves `spare_sms` SMs to the work that runs beside it. Records side->join.
static int launch_shared_side(const fm_layer* L, const uint16_t* xb, const float* sgate, int T, int t_real, float* out,
                              int* gu_list, int* dn_list, uint16_t* h_rows, int h_ld, int spare_sms, int* err,
                              SideStream* side, cudaStream_t st) {
    const int H = L->hidden, El = L->e_local;
    std::lock_guard<std::mutex> lock(side->enqueue);
    cudaStream_t s2 = side->s;
    if (cudaEventRecord(side->fork, st) != cudaSuccess || cudaStreamWaitEvent(s2, side->fork, 0) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "fork the shared expert");
    int rc = launch_seg_lists(nullptr, 0, El, 0, t_real, gu_list, L->ffn / 64, L->shared_ffn / 64, dn_list,
                              H / kTileRows, kBNTc, s2);
    if (rc) return rc;
    const int rt = (T + kBNTc - 1) / kBNTc;
    TcLaunch g{};
    g.max_items = rt * (L->shared_ffn / 64);
    g.max_ctas = spare_sms > 0 ? device_sm_count() - spare_sms : 0;
    g.list = gu_list;
    g.act = xb;
    g.act_rows = T;
    g.act_cols = H;
    g.act_ld = H;
    g.w_routed = L->gate_up;
    g.w_routed_stride = (size_t)2 * L->ffn * H / 32 * 20;
    g.w_shared = L->shared_gate_up;
    g.shared_group = El;
    g.K_routed = H;
    g.K_shared = H;
    g.h_out = h_rows;
    g.h_ld = h_ld;
    g.err = err;
    if ((rc = launch_expert_tc(true, g, s2))) return rc;
    TcLaunch d{};
    d.max_items = rt * (H / kTileRows);
    d.max_ctas = g.max_ctas;
    d.list = dn_list;
    d.act = h_rows;
    d.act_rows = T;
    d.act_cols = h_ld;
    d.act_ld = h_ld;
    d.w_routed = L->down;
    d.w_routed_stride = (size_t)H * L->ffn / 32 * 20;
    d.w_shared = L->shared_down;
    d.shared_group = El;
    d.K_routed = L->ffn;
    d.K_shared = L->shared_ffn;
    d.out = out;
    d.H = H;
    d.k = L->top_k;
    d.shared_base = 0;
    d.sgate = sgate;
    d.err = err;
    if ((rc = launch_expert_tc(false, d, s2))) return rc;
    if (cudaEventRecord(side->join, s2) != cudaSuccess) return cuda_status(cudaGetLastError(), "join event");
    return FM_OK;
}

static int run_block(const fm_layer* L, const uint16_t* xb, const float* res, const int32_t* idx, const float* w,
                     const float* sgate, int T, int t_real, float* out, void* ws, const Layout& lo, cudaStream_t st) {
    const int H = L->hidden, k = L->top_k, E = L->n_experts;
    const bool shared_on = L->shared_ffn > 0 && sgate && L->shared_gate_up && L->shared_down && t_real > 0;
    if (pick_path(L, T) == Path::Gemv) return run_block_gemv(L, xb, res, idx, w, sgate, T, t_real, out, ws, lo, st);
    const int P = t_real * k;
    // (the caller cleared the status words before this call's first kernel: clear_status)
    const int nblk = (P + kChunk - 1) / kChunk;
    // rows of the sorted space: routed [0, P), shared [P_cap, P_cap + t_real) with P_cap = T * k
    const int Pcap = lo.P;
    // the shared expert reads x directly and runs on a side stream while the routed rows are dispatched
    // and gathered (those kernels leave most SMs idle); out = res must precede it. In the fixed-order mode
    // the down GEMM writes every y row (shared rows too, as one more group) and the combine kernel sums
    // each token's terms in ascending expert order, writing all of out.
    const bool fixed = fixed_order(L);
    const bool shared_in_lists = shared_on && fixed;
    SideStream* side = (shared_on && !fixed) ? side_stream() : nullptr;
    if (shared_on && !fixed && !side) {
        set_error("could not create the side stream");
        return FM_ECUDA;
    }
    int rc = FM_OK;
    if (!fixed && cudaMemcpyAsync(out, res, (size_t)T * H * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "out = res");
    if (side && (rc = launch_shared_side(L, xb, sgate, T, t_real, out, at<int>(ws, lo.gu_list_sh),
                                         at<int>(ws, lo.dn_list_sh), at<uint16_t>(ws, lo.hperm) + (size_t)Pcap * lo.fmax,
                                         lo.fmax, 0, at<int>(ws, lo.err) + 1, side, st)))
        return rc;
    prof_begin(kStageDispatch, st);
    rc = launch_dispatch(idx, P, L->e_begin, L->e_local, E, Pcap, shared_in_lists ? t_real : 0, at<int>(ws, lo.blk_hist),
                         nblk, at<int>(ws, lo.counts), at<int>(ws, lo.offsets), at<int>(ws, lo.pos),
                         at<int>(ws, lo.pair), at<int>(ws, lo.gu_list), L->ffn / 64,
                         shared_in_lists ? L->shared_ffn / 64 : 0, at<int>(ws, lo.dn_list), H / kTileRows, kBNTc,
                         at<int>(ws, lo.err), st);
    if (rc) return rc;
    prof_end(kStageDispatch, st);
    prof_begin(kStageGather, st);
    if ((rc = launch_gather(xb, at<int>(ws, lo.pair), at<int>(ws, lo.counts), at<int>(ws, lo.offsets), L->e_local, Pcap,
                            k, H, lo.rows, at<uint16_t>(ws, lo.xperm), st)))
        return rc;
    prof_end(kStageGather, st);
    // out = res was set above (rows past t_real stay res); the down GEMM adds w * y into it (or, in the
    // fixed-order mode, writes the y rows the combine then sums)
    TcLaunch g{};
    g.max_items = lo.max_gu;
    g.list = at<int>(ws, lo.gu_list);
    g.act = at<uint16_t>(ws, lo.xperm);
    g.act_rows = lo.rows;
    g.act_cols = H;
    g.act_ld = H;
    g.w_routed = L->gate_up;
    g.w_routed_stride = (size_t)2 * L->ffn * H / 32 * 20;
    g.w_shared = L->shared_gate_up;
    g.shared_group = L->e_local;
    g.K_routed = H;
    g.K_shared = H;
    g.h_out = at<uint16_t>(ws, lo.hperm);
    g.h_ld = lo.fmax;
    g.err = at<int>(ws, lo.err) + 1;
    prof_begin(kStageGateUp, st);
    if ((rc = launch_expert_tc(true, g, st))) return rc;
    prof_end(kStageGateUp, st);
    TcLaunch d{};
    d.max_items = lo.max_dn;
    d.list = at<int>(ws, lo.dn_list);
    d.act = at<uint16_t>(ws, lo.hperm);
    d.act_rows = lo.rows;
    d.act_cols = lo.fmax;
    d.act_ld = lo.fmax;
    d.w_routed = L->down;
    d.w_routed_stride = (size_t)H * L->ffn / 32 * 20;
    d.w_shared = L->shared_down;
    d.shared_group = L->e_local;
    d.K_routed = L->ffn;
    d.K_shared = L->shared_ffn;
    d.out = out;
    d.H = H;
    d.pair = at<int>(ws, lo.pair);
    d.wpair = w;
    d.k = k;
    d.shared_base = Pcap;
    d.sgate = sgate;
    d.err = at<int>(ws, lo.err) + 1;
    d.y_f32 = fixed ? at<float>(ws, lo.yperm) : nullptr;
    prof_begin(kStageDown, st);
    if ((rc = launch_expert_tc(false, d, st))) return rc;
    prof_end(kStageDown, st);
    if (side && cudaStreamWaitEvent(st, side->join, 0) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "join the shared expert");
    if (fixed) {
        prof_begin(kStageCombine, st);
        rc = launch_combine(res, at<float>(ws, lo.yperm), at<int>(ws, lo.pos), idx, w, sgate, shared_on ? 1 : 0, T,
                            t_real, k, H, Pcap, out, st);
        prof_end(kStageCombine, st);
        if (rc) return rc;
    }
    return FM_OK;
}

}  // namespace fm

using namespace fm;

extern "C" FM_API int fm_last_error(char* buf, size_t n) {
    if (buf && n) {
        std::strncpy(buf, g_err, n - 1);
        buf[n - 1] = 0;
    }
    return FM_OK;
}

extern "C" FM_API int fm_version(char* buf, size_t n) {
    if (buf && n) std::snprintf(buf, n, "flowmoe 0.1 sm_100a");
    return FM_OK;
}

extern "C" FM_API int fm_workspace_size(const fm_layer* L, int32_t T, size_t* bytes) {
    g_err[0] = 0;
    if (int rc = validate(L, T)) return rc;
    *bytes = make_layout(L, T).total;
    return FM_OK;
}

extern "C" FM_API int fm_router_topk(const fm_layer* L, const void* xm, int32_t xm_dtype, int32_t T, float* probs,
                              int32_t* idx, float* w, float* shared_gate, void* workspace, size_t workspace_bytes,
                              void* stream) {
    g_err[0] = 0;
    if (int rc = validate(L, T)) return rc;
    if (T == 0) return FM_OK;
    const Layout lo = make_layout(L, T);
    if (int rc = check_ws(lo, workspace, workspace_bytes)) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    if (int rc = clear_status(workspace, lo, st)) return rc;
    const uint16_t* xb = nullptr;
    if (int rc = xm_to_bf16(L, xm, xm_dtype, T, workspace, lo, &xb, st)) return rc;
    return launch_router(xb, L->router, L->router_bias, T, L->hidden, L->n_experts, L->top_k, fixed_order(L), at<float>(workspace, lo.logits), probs,
                         idx, w, shared_gate, at<int>(workspace, lo.err), st);
}

extern "C" FM_API int fm_moe_block(const fm_layer* L, const void* xm, int32_t xm_dtype, const float* res, const int32_t* idx,
                            const float* w, const float* shared_gate, int32_t T, int32_t t_real, float* out,
                            void* workspace, size_t workspace_bytes, void* stream) {
    g_err[0] = 0;
    if (int rc = validate(L, T)) return rc;
    if (t_real < 0 || t_real > T) {
        set_error("t_real %d outside [0, T=%d]", t_real, T);
        return FM_EINVAL_SHAPE;
    }
    if (T == 0) return FM_OK;
    const Layout lo = make_layout(L, T);
    if (int rc = check_ws(lo, workspace, workspace_bytes)) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    const uint16_t* xb = nullptr;
    if (pick_path(L, T) == Path::Tc || fixed_order(L))   // else the GEMV path's dispatch kernel clears them
        if (int rc = clear_status(workspace, lo, st)) return rc;
    if (int rc = xm_to_bf16(L, xm, xm_dtype, T, workspace, lo, &xb, st)) return rc;
    return run_block(L, xb, res, idx, w, shared_gate, T, t_real, out, workspace, lo, st);
}

namespace fm {
// Router + shared expert + experts over bf16 activations xb (shared by fm_moe_layer and
// fm_moe_layer_norm).
static int moe_layer_xb(const fm_layer* L, const uint16_t* xb, const float* res, int T, int t_real, float* out,
                        int32_t* idx, float* w, void* workspace, const Layout& lo, cudaStream_t st) {
    int32_t* ids = idx ? idx : at<int32_t>(workspace, lo.idx);
    float* ws_w = w ? w : at<float>(workspace, lo.w);
    float* sg = at<float>(workspace, lo.sgate);
    if (pick_path(L, T) == Path::Tc || fixed_order(L))   // else the GEMV path's dispatch kernel clears them
        if (int rc = clear_status(workspace, lo, st)) return rc;
    prof_begin(kStageRouter, st);
    if (int rc = launch_router(xb, L->router, L->router_bias, T, L->hidden, L->n_experts, L->top_k, fixed_order(L),
                               at<float>(workspace, lo.logits), nullptr, ids, ws_w, sg, at<int>(workspace, lo.err), st))
        return rc;
    prof_end(kStageRouter, st);
    return run_block(L, xb, res, ids, ws_w, sg, T, t_real, out, workspace, lo, st);
}
}  // namespace fm

extern "C" FM_API int fm_moe_layer_norm(const fm_layer* L, const float* x, const uint16_t* norm_w, float eps, int32_t T,
                                        int32_t t_real, float* out, int32_t* idx, float* w, void* workspace,
                                        size_t workspace_bytes, void* stream) {
    g_err[0] = 0;
    if (int rc = validate(L, T)) return rc;
    if (t_real < 0 || t_real > T || !norm_w || !(eps >= 0.f)) {
        set_error("t_real %d outside [0, T=%d], or no norm weight / a negative eps", t_real, T);
        return FM_EINVAL_SHAPE;
    }
    if (T == 0) return FM_OK;
    const Layout lo = make_layout(L, T);
    if (int rc = check_ws(lo, workspace, workspace_bytes)) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    uint16_t* xb = at<uint16_t>(workspace, lo.xb);
    prof_begin(kStageToBf16, st);
    if (int rc = launch_rmsnorm_bf16(x, norm_w, eps, T, L->hidden, xb, st)) return rc;
    prof_end(kStageToBf16, st);
    return moe_layer_xb(L, xb, x, T, t_real, out, idx, w, workspace, lo, st);
}

extern "C" FM_API int fm_rmsnorm_bf16(const float* x, const uint16_t* norm_w, float eps, int32_t T, int32_t H,
                                       uint16_t* xb, void* stream) {
    g_err[0] = 0;
    if (T < 0 || H <= 0 || H % 4 || !(eps >= 0.f) || (T > 0 && (!x || !norm_w || !xb))) {
        set_error("fm_rmsnorm_bf16: T=%d H=%d (H %% 4 == 0), eps, and non-null buffers needed", T, H);
        return FM_EINVAL_SHAPE;
    }
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(norm_w) & 7) ||
        (reinterpret_cast<uintptr_t>(xb) & 7)) {
        set_error("fm_rmsnorm_bf16: x must be 16-byte aligned, norm_w and xb 8-byte aligned");
        return FM_EINVAL_SHAPE;
    }
    return launch_rmsnorm_bf16(x, norm_w, eps, T, H, xb, (cudaStream_t)stream);
}

extern "C" FM_API int fm_moe_layer(const fm_layer* L, const void* xm, int32_t xm_dtype, const float* res, int32_t T,
                            int32_t t_real, float* out, int32_t* idx, float* w, void* workspace, size_t workspace_bytes,
                            void* stream) {
    g_err[0] = 0;
    if (int rc = validate(L, T)) return rc;
    if (t_real < 0 || t_real > T) {
        set_error("t_real %d outside [0, T=%d]", t_real, T);
        return FM_EINVAL_SHAPE;
    }
    if (T == 0) return FM_OK;
    const Layout lo = make_layout(L, T);
    if (int rc = check_ws(lo, workspace, workspace_bytes)) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    const uint16_t* xb = nullptr;
    if (int rc = xm_to_bf16(L, xm, xm_dtype, T, workspace, lo, &xb, st)) return rc;
    return moe_layer_xb(L, xb, res, T, t_real, out, idx, w, workspace, lo, st);
}

extern "C" FM_API int fm_moe_dispatch(const fm_layer* L, const int32_t* idx, int32_t T, int32_t t_real, int32_t* counts,
                                       int32_t* offsets, int32_t* pos, int32_t* pair, void* workspace,
                                       size_t workspace_bytes, void* stream) {
    g_err[0] = 0;
    if (int rc = validate(L, T)) return rc;
    if (t_real < 0 || t_real > T) {
        set_error("t_real %d outside [0, T=%d]", t_real, T);
        return FM_EINVAL_SHAPE;
    }
    if (T == 0) return FM_OK;
    const Layout lo = make_layout(L, T);
    if (int rc = check_ws(lo, workspace, workspace_bytes)) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    const int k = L->top_k, P = t_real * k, nblk = (P + kChunk - 1) / kChunk;
    if (cudaMemsetAsync(at<int>(workspace, lo.err), 0, 16, st) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "memset");
    if (int rc = launch_dispatch(idx, P, L->e_begin, L->e_local, L->n_experts, lo.P, 0, at<int>(workspace, lo.blk_hist),
                                 nblk, at<int>(workspace, lo.counts), at<int>(workspace, lo.offsets),
                                 at<int>(workspace, lo.pos), at<int>(workspace, lo.pair), at<int>(workspace, lo.gu_list),
                                 L->ffn / kTileRows, 0, at<int>(workspace, lo.dn_list), L->hidden / kTileRows, kBN,
                                 at<int>(workspace, lo.err), st))
        return rc;
    const size_t E = (size_t)L->e_local;
    cudaError_t e = cudaSuccess;
    if (counts && e == cudaSuccess) e = cudaMemcpyAsync(counts, at<int>(workspace, lo.counts), E * 4, cudaMemcpyDeviceToDevice, st);
    if (offsets && e == cudaSuccess)
        e = cudaMemcpyAsync(offsets, at<int>(workspace, lo.offsets), (E + 1) * 4, cudaMemcpyDeviceToDevice, st);
    if (pos && P && e == cudaSuccess) e = cudaMemcpyAsync(pos, at<int>(workspace, lo.pos), (size_t)P * 4, cudaMemcpyDeviceToDevice, st);
    if (pair && P && e == cudaSuccess) e = cudaMemcpyAsync(pair, at<int>(workspace, lo.pair), (size_t)P * 4, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_status(e, "copy dispatch results");
    return FM_OK;
}

extern "C" FM_API int fm_launch_count(unsigned long long* n) {
    *n = g_launches.load(std::memory_order_relaxed);
    return FM_OK;
}

extern "C" FM_API int fm_profile(int32_t enable) {
    g_err[0] = 0;
    if (enable && !g_prof.ev[0][0]) {
        for (auto& p : g_prof.ev)
            for (auto& e : p)
                if (cudaEventCreate(&e) != cudaSuccess) return cuda_status(cudaGetLastError(), "cudaEventCreate");
    }
    g_prof.on = enable != 0;
    g_prof.n = 0;
    for (int& o : g_prof.open) o = -1;
    return FM_OK;
}

extern "C" FM_API int fm_profile_read(double* ms, int32_t n_stages) {
    g_err[0] = 0;
    for (int i = 0; i < n_stages; ++i) ms[i] = 0.0;
    for (int i = 0; i < g_prof.n; ++i) {
        float t = 0.f;
        if (cudaEventSynchronize(g_prof.ev[i][1]) != cudaSuccess) return cuda_status(cudaGetLastError(), "event sync");
        if (cudaEventElapsedTime(&t, g_prof.ev[i][0], g_prof.ev[i][1]) != cudaSuccess)
            return cuda_status(cudaGetLastError(), "event elapsed");
        if (g_prof.stage[i] < n_stages) ms[g_prof.stage[i]] += t;
    }
    g_prof.n = 0;
    return FM_OK;
}

extern "C" FM_API int fm_moe_check(void* workspace, void* stream) {
    g_err[0] = 0;
    int word[2] = {0, 0};   // the error words sit at the start of every workspace layout
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaStreamSynchronize(st) != cudaSuccess) return cuda_status(cudaGetLastError(), "stream sync");
    if (cudaMemcpy(word, workspace, sizeof(word), cudaMemcpyDeviceToHost) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "read error words");
    if (word[1] == FM_EINVAL_SHAPE) {
        set_error("expert parallel: the received row counts are negative or do not add up to R; no rows were computed");
        return word[1];
    }
    if (word[1]) {
        set_error("a device wait gave up (status %d): the block's output is incomplete", word[1]);
        return word[1];
    }
    if (word[0]) {
        set_error("router produced %d expert index(es) outside the experts this block holds", word[0]);
        return FM_EINVAL_EXPERT;
    }
    return FM_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// Expert parallel: three device stages around the host's two all-to-all exchanges (see flowmoe/ep.py).
//   fm_ep_dispatch  router + stable sort over ALL experts + gather: the rows bound for rank g are the
//                   contiguous expert range [g * e_local, (g + 1) * e_local) of the sorted matrix;
//   fm_ep_experts   the rows received from every rank regrouped expert-major, this rank's experts
//                   (tcgen05 grouped GEMMs) written back as unweighted bf16 rows in the received order,
//                   and the replicated shared expert of this rank's own tokens added into out = res;
//   fm_ep_combine   out[t] += w * y for t's pairs, y the rows the expert ranks returned.
namespace fm {

struct EpDispatchLayout {
    size_t err, logits, counts, offsets, blk_hist, pair, gu_list, dn_list, total;
    int P, nblk;
};

static EpDispatchLayout ep_dispatch_layout(const fm_layer* L, int T) {
    EpDispatchLayout o{};
    const int H = L->hidden, E = L->n_experts, k = L->top_k;
    o.P = T * k;
    o.nblk = (o.P + kChunk - 1) / kChunk;
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t a = off; off = align256(off + bytes); return a; };
    o.err = take(16);
    o.logits = take(router_scratch_bytes(T, H, E, fixed_order(L)));
    o.counts = take((size_t)(E + 1) * 4);
    o.offsets = take((size_t)(E + 2) * 4);
    o.blk_hist = take((size_t)o.nblk * E * 4);
    o.pair = take((size_t)o.P * 4);
    o.gu_list = take(16);
    o.dn_list = take(16);
    o.total = off;
    return o;
}

struct EpExpertsLayout {
    size_t err, seg, src_off, dst_off, rowmap, gu_list, dn_list, xexp, hexp, total;
    int rows, fmax, max_gu, max_dn;
};

static EpExpertsLayout ep_experts_layout(const fm_layer* L, int T, int R, int G) {
    EpExpertsLayout o{};
    const int H = L->hidden, El = L->e_local;
    o.rows = R + T;
    o.fmax = L->ffn > L->shared_ffn ? L->ffn : L->shared_ffn;
    const int rt_routed = R / kBNTc + El;
    const int rt_shared = (T + kBNTc - 1) / kBNTc;
    o.max_gu = rt_routed * (L->ffn / 64) + rt_shared * (L->shared_ffn / 64);
    o.max_dn = (rt_routed + (L->shared_ffn ? rt_shared : 0)) * (H / kTileRows);
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t a = off; off = align256(off + bytes); return a; };
    o.err = take(16);
    o.seg = take((size_t)El * 3 * 4);
    o.src_off = take((size_t)G * El * 4);
    o.dst_off = take((size_t)G * El * 4);
    o.rowmap = take((size_t)(R > 0 ? R : 1) * 4);
    o.gu_list = take((size_t)(4 + 4 * o.max_gu) * 4);
    o.dn_list = take((size_t)(4 + 4 * o.max_dn) * 4);
    o.xexp = take((size_t)o.rows * H * 2);
    o.hexp = take((size_t)o.rows * o.fmax * 2);
    o.total = off;
    return o;
}

static int ep_check(const fm_layer* L, int T, int R, int G) {
    if (int rc = validate(L, T)) return rc;
    if (G <= 0 || R < 0 || L->e_local <= 0 || L->e_local > 1024 || (size_t)G * L->e_local > (1u << 20)) {
        set_error("expert parallel: bad n_ranks %d / received rows %d / local experts %d (1..1024)", G, R, L->e_local);
        return FM_EINVAL_SHAPE;
    }
    return FM_OK;
}

static int ws_ok(size_t need, void* ws, size_t bytes) {
    if (!ws || bytes < need) {
        set_error("workspace of %zu B is smaller than the %zu B needed", bytes, need);
        return FM_EWORKSPACE;
    }
    if (reinterpret_cast<uintptr_t>(ws) & 255) {
        set_error("workspace must be 256-byte aligned");
        return FM_EWORKSPACE;
    }
    return FM_OK;
}

}  // namespace fm

extern "C" FM_API int fm_ep_workspace_size(const fm_layer* L, int32_t T, int32_t R, int32_t n_ranks, size_t* bytes) {
    g_err[0] = 0;
    if (int rc = ep_check(L, T, R, n_ranks)) return rc;
    const size_t a = ep_dispatch_layout(L, T).total, b = ep_experts_layout(L, T, R, n_ranks).total;
    *bytes = a > b ? a : b;
    return FM_OK;
}

extern "C" FM_API int fm_ep_dispatch(const fm_layer* L, const void* xm, int32_t xm_dtype, int32_t T, int32_t t_real,
                                     uint16_t* xb_out, int32_t* idx, float* w, float* shared_gate, int32_t* counts,
                                     int32_t* pos, uint16_t* xsend, void* workspace, size_t workspace_bytes,
                                     void* stream) {
    g_err[0] = 0;
    if (int rc = validate(L, T)) return rc;
    if (t_real < 0 || t_real > T) {
        set_error("t_real %d outside [0, T=%d]", t_real, T);
        return FM_EINVAL_SHAPE;
    }
    const int H = L->hidden, E = L->n_experts, k = L->top_k;
    cudaStream_t st = (cudaStream_t)stream;
    if (T == 0) {
        if (cudaMemsetAsync(counts, 0, (size_t)E * 4, st) != cudaSuccess) return cuda_status(cudaGetLastError(), "memset");
        return FM_OK;
    }
    const EpDispatchLayout lo = ep_dispatch_layout(L, T);
    if (int rc = ws_ok(lo.total, workspace, workspace_bytes)) return rc;
    const uint16_t* xb = static_cast<const uint16_t*>(xm);
    if (xm_dtype == FM_F32) {
        if (!xb_out) {
            set_error("fm_ep_dispatch: f32 activations need xb_out for their bf16 copy");
            return FM_EINVAL_SHAPE;
        }
        prof_begin(kStageToBf16, st);
        if (int rc = launch_to_bf16(static_cast<const float*>(xm), xb_out, (long long)T * H, st)) return rc;
        prof_end(kStageToBf16, st);
        xb = xb_out;
    } else if (xm_dtype != FM_BF16) {
        set_error("xm dtype %d is neither FM_F32 nor FM_BF16", xm_dtype);
        return FM_EINVAL_SHAPE;
    }
    if (cudaMemsetAsync(at<int>(workspace, lo.err), 0, 16, st) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "memset");
    prof_begin(kStageRouter, st);
    if (int rc = launch_router(xb, L->router, L->router_bias, T, H, E, k, fixed_order(L), at<float>(workspace, lo.logits), nullptr, idx, w,
                               shared_gate, at<int>(workspace, lo.err), st))
        return rc;
    prof_end(kStageRouter, st);
    const int P = t_real * k;
    prof_begin(kStageDispatch, st);
    int rc = launch_dispatch(idx, P, 0, E, E, lo.P, 0, at<int>(workspace, lo.blk_hist), (P + kChunk - 1) / kChunk,
                             at<int>(workspace, lo.counts), at<int>(workspace, lo.offsets), pos,
                             at<int>(workspace, lo.pair), at<int>(workspace, lo.gu_list), 0, 0,
                             at<int>(workspace, lo.dn_list), 0, kBNTc, at<int>(workspace, lo.err), st);
    if (rc) return rc;
    if (cudaMemcpyAsync(counts, at<int>(workspace, lo.counts), (size_t)E * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "counts copy");
    prof_end(kStageDispatch, st);
    prof_begin(kStageGather, st);
    rc = launch_gather(xb, at<int>(workspace, lo.pair), at<int>(workspace, lo.counts), at<int>(workspace, lo.offsets), E,
                       lo.P, k, H, P, xsend, st);
    prof_end(kStageGather, st);
    return rc;
}

extern "C" FM_API int fm_ep_experts(const fm_layer* L, const uint16_t* xrecv, int32_t R, const int32_t* recv_counts,
                                    int32_t n_ranks, const uint16_t* xb, const float* shared_gate, const float* res,
                                    int32_t T, int32_t t_real, float* out, uint16_t* yrecv, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    g_err[0] = 0;
    if (int rc = ep_check(L, T, R, n_ranks)) return rc;
    if (t_real < 0 || t_real > T) {
        set_error("t_real %d outside [0, T=%d]", t_real, T);
        return FM_EINVAL_SHAPE;
    }
    if (T == 0 && R == 0) return FM_OK;
    const int H = L->hidden, El = L->e_local;
    const EpExpertsLayout lo = ep_experts_layout(L, T, R, n_ranks);
    if (int rc = ws_ok(lo.total, workspace, workspace_bytes)) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    const bool shared_on = L->shared_ffn > 0 && L->shared_gate_up && L->shared_down && shared_gate && t_real > 0;
    const int srows = shared_on ? t_real : 0;
    if (cudaMemsetAsync(at<int>(workspace, lo.err), 0, 16, st) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "memset");
    if (T > 0 && cudaMemcpyAsync(out, res, (size_t)T * H * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "out = res");
    prof_begin(kStageGather, st);
    int rc = launch_ep_regroup(recv_counts, n_ranks, El, xrecv, R, xb, srows, H, at<int>(workspace, lo.seg),
                               at<int>(workspace, lo.src_off), at<int>(workspace, lo.dst_off),
                               at<uint16_t>(workspace, lo.xexp), at<int>(workspace, lo.rowmap),
                               at<int>(workspace, lo.err), st);
    if (rc) return rc;
    prof_end(kStageGather, st);
    prof_begin(kStageDispatch, st);
    rc = launch_seg_lists(at<int>(workspace, lo.seg), El, El, R, srows, at<int>(workspace, lo.gu_list),
                          L->ffn / 64, L->shared_ffn / 64, at<int>(workspace, lo.dn_list),
                          H / kTileRows, kBNTc, st);
    if (rc) return rc;
    prof_end(kStageDispatch, st);
    TcLaunch g{};
    g.max_items = lo.max_gu;
    g.list = at<int>(workspace, lo.gu_list);
    g.act = at<uint16_t>(workspace, lo.xexp);
    g.act_rows = lo.rows;
    g.act_cols = H;
    g.act_ld = H;
    g.w_routed = L->gate_up;
    g.w_routed_stride = (size_t)2 * L->ffn * H / 32 * 20;
    g.w_shared = L->shared_gate_up;
    g.shared_group = El;
    g.K_routed = H;
    g.K_shared = H;
    g.h_out = at<uint16_t>(workspace, lo.hexp);
    g.h_ld = lo.fmax;
    g.err = at<int>(workspace, lo.err) + 1;
    prof_begin(kStageGateUp, st);
    if ((rc = launch_expert_tc(true, g, st))) return rc;
    prof_end(kStageGateUp, st);
    TcLaunch d{};
    d.max_items = lo.max_dn;
    d.list = at<int>(workspace, lo.dn_list);
    d.act = at<uint16_t>(workspace, lo.hexp);
    d.act_rows = lo.rows;
    d.act_cols = lo.fmax;
    d.act_ld = lo.fmax;
    d.w_routed = L->down;
    d.w_routed_stride = (size_t)H * L->ffn / 32 * 20;
    d.w_shared = L->shared_down;
    d.shared_group = El;
    d.K_routed = L->ffn;
    d.K_shared = L->shared_ffn;
    d.out = out;
    d.H = H;
    d.ymap = at<int>(workspace, lo.rowmap);
    d.k = L->top_k;
    d.shared_base = R;
    d.sgate = shared_gate;
    d.y_rows = yrecv;
    d.err = at<int>(workspace, lo.err) + 1;
    prof_begin(kStageDown, st);
    if ((rc = launch_expert_tc(false, d, st))) return rc;
    prof_end(kStageDown, st);
    return FM_OK;
}

extern "C" FM_API int fm_ep_combine(const fm_layer* L, float* out, const uint16_t* ysorted, const int32_t* pos,
                                    const int32_t* idx, const float* w, int32_t T, int32_t t_real, void* stream) {
    g_err[0] = 0;
    if (int rc = validate(L, T)) return rc;
    if (t_real < 0 || t_real > T) {
        set_error("t_real %d outside [0, T=%d]", t_real, T);
        return FM_EINVAL_SHAPE;
    }
    cudaStream_t st = (cudaStream_t)stream;
    prof_begin(kStageCombine, st);
    const int rc = launch_combine_bf16(out, ysorted, pos, idx, w, T, t_real, L->top_k, L->hidden, st);
    prof_end(kStageCombine, st);
    return rc;
}

// ---------------------------------------------------------------------------------------------------------------
// Expert parallel over peer memory (ep_peer.cu): fm_ep_peer_layer and the IPC helpers.
namespace fm {

struct EpSymLayout {
    size_t state, flags, cnt, meta, x, y, total;
    int r_cap;
};

static EpSymLayout ep_sym_layout(const fm_layer* L, const fm_ep_group* g) {
    EpSymLayout o{};
    const int H = L->hidden, E = L->n_experts, k = L->top_k, G = g->n_ranks;
    o.r_cap = G * g->t_cap * k;
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t a = off; off = align256(off + bytes); return a; };
    o.state = take(256);
    o.flags = take((size_t)3 * kMaxRanksPad * 4);
    o.cnt = take((size_t)G * E * 4);
    o.meta = take((size_t)o.r_cap * 4);
    o.x = take(((size_t)o.r_cap + g->t_cap) * H * 2);
    o.y = take((size_t)g->t_cap * k * H * 2 + 16);
    o.total = off;
    return o;
}

struct EpPeerLayout {
    size_t err, xb, logits, counts, offsets, blk_hist, pos, pair, idx, w, sgate, send_base, seg, gu_list, dn_list, hexp;
    size_t gu_list_sh, dn_list_sh;
    size_t total;
    int max_gu, max_dn, fmax, max_gu_sh, max_dn_sh;
};

static EpPeerLayout ep_peer_layout(const fm_layer* L, const fm_ep_group* g, int T) {
    EpPeerLayout o{};
    const int H = L->hidden, E = L->n_experts, k = L->top_k, El = L->e_local, tc = g->t_cap;
    const int r_cap = g->n_ranks * tc * k;
    const int P = T * k, nblk = (P + kChunk - 1) / kChunk;
    o.fmax = L->ffn > L->shared_ffn ? L->ffn : L->shared_ffn;
    const int rt_routed = r_cap / kBNTc + El, rt_shared = (tc + kBNTc - 1) / kBNTc;
    o.max_gu = rt_routed * (L->ffn / 64) + rt_shared * (L->shared_ffn / 64);
    o.max_dn = (rt_routed + (L->shared_ffn ? rt_shared : 0)) * (H / kTileRows);
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t a = off; off = align256(off + bytes); return a; };
    o.err = take(16);
    o.xb = take((size_t)T * H * 2);
    o.logits = take(router_scratch_bytes(T, H, E, fixed_order(L)));
    o.counts = take((size_t)(E + 1) * 4);
    o.offsets = take((size_t)(E + 2) * 4);
    o.blk_hist = take((size_t)nblk * E * 4);
    o.pos = take((size_t)P * 4);
    o.pair = take((size_t)P * 4);
    o.idx = take((size_t)P * 4);
    o.w = take((size_t)P * 4);
    o.sgate = take((size_t)T * 4);
    o.send_base = take((size_t)E * 4);
    o.seg = take((size_t)El * 3 * 4);
    o.gu_list = take((size_t)(4 + 4 * o.max_gu) * 4);
    o.dn_list = take((size_t)(4 + 4 * o.max_dn) * 4);
    o.hexp = take(((size_t)r_cap + tc) * o.fmax * 2);
    o.max_gu_sh = rt_shared * (L->shared_ffn / 64);
    o.max_dn_sh = L->shared_ffn ? rt_shared * (H / kTileRows) : 0;
    o.gu_list_sh = take((size_t)(4 + 4 * o.max_gu_sh) * 4);
    o.dn_list_sh = take((size_t)(4 + 4 * o.max_dn_sh) * 4);
    o.total = off;
    return o;
}

constexpr int kScatterSms = 20;   // SMs left to the row exchange while the shared expert runs

static int ep_group_check(const fm_layer* L, const fm_ep_group* g, bool need_sym = true) {
    if (int rc = validate(L, 0)) return rc;
    if (!g || g->n_ranks < 1 || g->n_ranks > FM_EP_MAX_RANKS || g->rank < 0 || g->rank >= g->n_ranks || g->t_cap < 1) {
        set_error("bad expert-parallel group (rank/n_ranks/t_cap; at most %d ranks)", FM_EP_MAX_RANKS);
        return FM_EINVAL_SHAPE;
    }
    const int G = g->n_ranks, E = L->n_experts;
    if (E % G || L->e_local != E / G || L->e_begin != g->rank * (E / G)) {
        set_error("expert-parallel layer must hold experts [%d, %d) of %d on rank %d of %d", g->rank * (E / G),
                  (g->rank + 1) * (E / G), E, g->rank, G);
        return FM_EINVAL_SHAPE;
    }
    if ((long long)g->t_cap * L->top_k >= (1ll << 24) || (long long)G * g->t_cap * L->top_k >= (1ll << 30)) {
        set_error("t_cap %d too large for the row metadata (t_cap * top_k < 2^24)", g->t_cap);
        return FM_EINVAL_SHAPE;
    }
    for (int i = 0; need_sym && i < G; ++i)
        if (!g->sym[i]) {
            set_error("expert-parallel group: rank %d's symmetric buffer is not mapped", i);
            return FM_EINVAL_SHAPE;
        }
    return FM_OK;
}


}  // namespace fm

extern "C" FM_API int fm_ep_peer_sizes(const fm_layer* L, const fm_ep_group* g, size_t* sym_bytes, size_t* ws_bytes) {
    g_err[0] = 0;
    if (int rc = ep_group_check(L, g, false)) return rc;
    if (sym_bytes) *sym_bytes = ep_sym_layout(L, g).total;
    if (ws_bytes) {
        size_t m = 0;   // the router's split-K scratch depends on T: the largest over 1..t_cap
        for (int T = 1; T <= g->t_cap; ++T) {
            const size_t t = ep_peer_layout(L, g, T).total;
            if (t > m) m = t;
        }
        *ws_bytes = m;
    }
    return FM_OK;
}

extern "C" FM_API int fm_ep_peer_layer(const fm_layer* L, const fm_ep_group* g, const void* xm, int32_t xm_dtype,
                                       const float* res, int32_t T, int32_t t_real, float* out, int32_t* idx, float* w,
                                       void* workspace, size_t workspace_bytes, void* stream) {
    g_err[0] = 0;
    if (int rc = ep_group_check(L, g)) return rc;
    if (int rc = validate(L, T)) return rc;
    if (T > g->t_cap || t_real < 0 || t_real > T) {
        set_error("T=%d / t_real=%d outside the group's t_cap %d", T, t_real, g->t_cap);
        return FM_EINVAL_SHAPE;
    }
    const int H = L->hidden, E = L->n_experts, k = L->top_k, El = L->e_local, G = g->n_ranks;
    const EpSymLayout sl = ep_sym_layout(L, g);
    const EpPeerLayout lo = ep_peer_layout(L, g, T);
    if (int rc = ws_ok(lo.total, workspace, workspace_bytes)) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    EpPeerArgs a{};
    for (int i = 0; i < G; ++i) a.sym[i] = static_cast<uint8_t*>(g->sym[i]);
    a.off_flags = sl.flags;
    a.off_cnt = sl.cnt;
    a.off_meta = sl.meta;
    a.off_x = sl.x;
    a.off_y = sl.y;
    a.state = reinterpret_cast<int*>(a.sym[g->rank] + sl.state);
    a.err = at<int>(workspace, lo.err);
    a.rank = g->rank;
    a.G = G;
    a.E = E;
    a.El = El;
    a.H = H;
    a.k = k;
    a.r_cap = sl.r_cap;
    a.timeout_ns = (long long)(g->timeout_ms > 0 ? g->timeout_ms : 10000) * 1000000ll;
    if (cudaMemsetAsync(a.err, 0, 16, st) != cudaSuccess) return cuda_status(cudaGetLastError(), "memset");
    const uint16_t* xb = static_cast<const uint16_t*>(xm);
    if (xm_dtype == FM_F32) {
        if (T > 0) {
            prof_begin(kStageToBf16, st);
            if (int rc = launch_to_bf16(static_cast<const float*>(xm), at<uint16_t>(workspace, lo.xb), (long long)T * H, st))
                return rc;
            prof_end(kStageToBf16, st);
        }
        xb = at<uint16_t>(workspace, lo.xb);
    } else if (xm_dtype != FM_BF16) {
        set_error("xm dtype %d is neither FM_F32 nor FM_BF16", xm_dtype);
        return FM_EINVAL_SHAPE;
    }
    int32_t* ids = idx ? idx : at<int32_t>(workspace, lo.idx);
    float* wts = w ? w : at<float>(workspace, lo.w);
    float* sg = at<float>(workspace, lo.sgate);
    const bool shared_on = L->shared_ffn > 0 && L->shared_gate_up && L->shared_down && t_real > 0;
    const int P = t_real * k;
    int rc = FM_OK;
    prof_begin(kStageRouter, st);
    if (T > 0 && (rc = launch_router(xb, L->router, L->router_bias, T, H, E, k, fixed_order(L), at<float>(workspace, lo.logits), nullptr,
                                     ids, wts, sg, a.err, st)))
        return rc;
    prof_end(kStageRouter, st);
    prof_begin(kStageDispatch, st);
    int* counts = at<int>(workspace, lo.counts);
    int* offsets = at<int>(workspace, lo.offsets);
    if ((rc = launch_dispatch(ids, P, 0, E, E, T * k, 0, at<int>(workspace, lo.blk_hist), (P + kChunk - 1) / kChunk,
                              counts, offsets, at<int>(workspace, lo.pos), at<int>(workspace, lo.pair),
                              at<int>(workspace, lo.gu_list), 0, 0, at<int>(workspace, lo.dn_list), 0, kBNTc, a.err, st)))
        return rc;
    // out = res before the fork: the shared expert adds into it on the side stream
    if (T > 0 && cudaMemcpyAsync(out, res, (size_t)T * H * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "out = res");
    // The shared expert needs no exchange: it runs on a side stream over this rank's own bf16 rows, on
    // all SMs but kScatterSms, while the rows travel; the combine waits for it (both add into out).
    SideStream* side = shared_on ? side_stream() : nullptr;
    if (shared_on && !side) {
        set_error("expert parallel: could not create the side stream");
        return FM_ECUDA;
    }
    if (shared_on && (rc = launch_shared_side(L, xb, sg, T, t_real, out, at<int>(workspace, lo.gu_list_sh),
                                              at<int>(workspace, lo.dn_list_sh),
                                              at<uint16_t>(workspace, lo.hexp) + (size_t)sl.r_cap * lo.fmax, lo.fmax,
                                              kScatterSms, a.err + 1, side, st)))
        return rc;
    if ((rc = launch_ep_post_counts(a, counts, st))) return rc;
    if ((rc = launch_ep_plan_peer(a, at<int>(workspace, lo.send_base), at<int>(workspace, lo.seg), st))) return rc;
    if ((rc = launch_seg_lists(at<int>(workspace, lo.seg), El, El, sl.r_cap, 0, at<int>(workspace, lo.gu_list),
                               L->ffn / 64, L->shared_ffn / 64, at<int>(workspace, lo.dn_list),
                               H / kTileRows, kBNTc, st)))
        return rc;
    prof_end(kStageDispatch, st);
    prof_begin(kStageGather, st);
    if ((rc = launch_ep_scatter_rows(a, xb, at<int>(workspace, lo.pair), ids, offsets, at<int>(workspace, lo.send_base), P,
                                     0, device_sm_count(), st)))
        return rc;
    if ((rc = launch_ep_wait(a, 1, st))) return rc;
    prof_end(kStageGather, st);
    uint8_t* mine = a.sym[g->rank];
    TcLaunch gu{};
    gu.max_items = lo.max_gu;
    gu.list = at<int>(workspace, lo.gu_list);
    gu.act = reinterpret_cast<const uint16_t*>(mine + sl.x);
    gu.act_rows = sl.r_cap + g->t_cap;
    gu.act_cols = H;
    gu.act_ld = H;
    gu.w_routed = L->gate_up;
    gu.w_routed_stride = (size_t)2 * L->ffn * H / 32 * 20;
    gu.w_shared = L->shared_gate_up;
    gu.shared_group = El;
    gu.K_routed = H;
    gu.K_shared = H;
    gu.h_out = at<uint16_t>(workspace, lo.hexp);
    gu.h_ld = lo.fmax;
    gu.err = a.err + 1;
    prof_begin(kStageGateUp, st);
    if ((rc = launch_expert_tc(true, gu, st))) return rc;
    prof_end(kStageGateUp, st);
    TcLaunch d{};
    d.max_items = lo.max_dn;
    d.list = at<int>(workspace, lo.dn_list);
    d.act = at<uint16_t>(workspace, lo.hexp);
    d.act_rows = sl.r_cap + g->t_cap;
    d.act_cols = lo.fmax;
    d.act_ld = lo.fmax;
    d.w_routed = L->down;
    d.w_routed_stride = (size_t)H * L->ffn / 32 * 20;
    d.w_shared = L->shared_down;
    d.shared_group = El;
    d.K_routed = L->ffn;
    d.K_shared = L->shared_ffn;
    d.out = out;
    d.H = H;
    d.k = k;
    d.shared_base = sl.r_cap;
    d.sgate = sg;
    d.meta = reinterpret_cast<const int*>(mine + sl.meta);
    for (int i = 0; i < G; ++i) d.yret[i] = reinterpret_cast<uint16_t*>(a.sym[i] + sl.y);
    d.err = a.err + 1;
    prof_begin(kStageDown, st);
    if ((rc = launch_expert_tc(false, d, st))) return rc;
    if ((rc = launch_ep_signal(a, 2, st))) return rc;
    prof_end(kStageDown, st);
    prof_begin(kStageCombine, st);
    if ((rc = launch_ep_wait(a, 2, st))) return rc;
    if (shared_on && cudaStreamWaitEvent(st, side->join, 0) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "join the shared expert");
    rc = launch_combine_bf16(out, reinterpret_cast<const uint16_t*>(mine + sl.y), at<int>(workspace, lo.pos), ids, wts, T,
                             t_real, k, H, st);
    prof_end(kStageCombine, st);
    return rc;
}

extern "C" FM_API int fm_ipc_alloc(size_t bytes, void** ptr, void* handle_out) {
    g_err[0] = 0;
    if (!ptr || !handle_out || !bytes) {
        set_error("fm_ipc_alloc: null argument or zero size");
        return FM_EINVAL_SHAPE;
    }
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return cuda_status(cudaGetLastError(), "cudaMalloc(symmetric buffer)");
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p);
        return cuda_status(cudaGetLastError(), "clear symmetric buffer");
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return cuda_status(cudaGetLastError(), "cudaIpcGetMemHandle");
    }
    std::memcpy(handle_out, &h, sizeof h);
    *ptr = p;
    return FM_OK;
}

extern "C" FM_API int fm_ipc_open(const void* handle, void** ptr) {
    g_err[0] = 0;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
        return cuda_status(cudaGetLastError(), "cudaIpcOpenMemHandle");
    return FM_OK;
}

extern "C" FM_API int fm_ipc_close(void* ptr) {
    g_err[0] = 0;
    if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) return cuda_status(cudaGetLastError(), "cudaIpcCloseMemHandle");
    return FM_OK;
}

extern "C" FM_API int fm_ipc_free(void* ptr) {
    g_err[0] = 0;
    if (cudaFree(ptr) != cudaSuccess) return cuda_status(cudaGetLastError(), "cudaFree(symmetric buffer)");
    return FM_OK;
}
