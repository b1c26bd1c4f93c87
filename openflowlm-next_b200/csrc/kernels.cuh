// Host-side launch wrappers of the kernels (router.cu, dispatch.cu, combine.cu, decode.cu, expert_tc.cu). Each returns an
// FM_* status and records the message with set_error on failure.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace fm {

int launch_to_bf16(const float* x, uint16_t* xb, long long n, cudaStream_t st);
int launch_rmsnorm_bf16(const float* x, const uint16_t* w, float eps, int T, int H, uint16_t* xb, cudaStream_t st);
// The router of T tokens (idx, w, sgate, optional probs): the logits into `logits`, from kRouterTcMinT
// tokens (E <= 496) by the tcgen05 kernel of router_tc.cu (row stride router_tc_ld(E); bounded waits
// report FM_ETIMEOUT in err[1]), below by the split-K logits kernel; then a top-k kernel. `fixed` (the
// fixed-order mode) takes one form at every T, so that a token's logits do not depend on the call's other
// tokens: the tcgen05 kernel where E <= 496, else one K chunk.
constexpr int kRouterTcMinT = 256;
bool router_tc_ok(int T, int E, int k, bool fixed);
int router_tc_ld(int E);
int launch_router(const uint16_t* xb, const uint16_t* router, const float* bias, int T, int H, int E, int k, bool fixed,
                  float* logits, float* probs, int32_t* idx, float* w, float* sgate, int* err, cudaStream_t st);
int launch_router_tc_logits(const uint16_t* xb, const uint16_t* router, int T, int H, int E, float* logits, int* err,
                            cudaStream_t st);
// The per-device side stream of the tcgen05 path (shared expert), created now if it does not exist yet.
int prepare_side_stream();
int launch_dispatch(const int32_t* idx, int P, int e_begin, int e_local, int E, int shared_base, int shared_rows,
                    int* blk_hist, int nblk,
                    int* counts, int* offsets, int* pos, int* pair, int* gu_list, int gu_bands, int gu_bands_shared,
                    int* dn_list, int dn_bands, int bn, int* err, cudaStream_t st);
int launch_gather(const uint16_t* xb, const int* pair, const int* counts, const int* offsets, int e_local, int shared_base,
                  int k, int H, int max_rows, uint16_t* xperm, cudaStream_t st);
// Most rows (tokens) of one tcgen05 work item: the MMA's N, one of the kernel's two TMEM accumulators.
constexpr int kTcItemRows = 256;
struct TcLaunch {
    int max_items;
    const int* list;
    const uint16_t* act;      // sorted bf16 activations (TMA source)
    int act_rows, act_cols, act_ld;
    const uint8_t* w_routed;
    size_t w_routed_stride;
    const uint8_t* w_shared;
    int shared_group;
    int K_routed, K_shared;
    uint16_t* h_out;          // GATE_UP
    int h_ld;
    float* out;               // DOWN
    int H;
    const int* pair;
    const float* wpair;
    int k;
    int shared_base;
    const float* sgate;
    uint16_t* y_rows;                // DOWN row mode (see expert_tc.cu)
    const int* ymap;
    float* y_f32;                    // DOWN f32 row mode (fixed-order combine)
    const int* meta;                 // peer expert-parallel DOWN (see expert_tc.cu)
    uint16_t* yret[kMaxRanks];
    int* err;
    int max_ctas;                    // grid cap (0: one CTA per SM); leaves SMs to concurrent work
};
int launch_expert_tc(bool gate_up, const TcLaunch& L, cudaStream_t st);
// bf16 matrix [rows, cols] (row stride ld elements) -> a TMA map with {64, box_rows} boxes, 128-byte swizzle.
int make_bmap(CUtensorMap* m, const uint16_t* base, int rows, int cols, int ld, int box_rows);
struct GemvLaunch {
    int max_items;
    const int* list;
    const uint8_t* w_routed;
    size_t w_routed_stride;
    const uint8_t* w_shared;
    int shared_group;
    int K_routed, K_shared;
    const uint16_t* act;
    int act_ld;
    const int* pair;
    int k;
    int shared_base;
    float* part;
    int part_rows, part_ld;
    int* done;
    uint16_t* h_out;
    int h_ld;
    int F_routed, F_shared;
    float* y_out;
    int H;
    const int* dn_list;   // GATE_UP: the down list (its K-chunk count)
    int y_rows;           // rows of y_out (cleared by GATE_UP when the down GEMM splits K)
    int* err;
    int tc_min;           // least token columns of an item's MMA (8 in the fixed-order mode)
};
int router_ksplit(int T, int H, int E, bool fixed);
size_t router_scratch_bytes(int T, int H, int E, bool fixed);   // the logits scratch of launch_router
int launch_dispatch_small(const int32_t* idx, int P, int e_begin, int e_local, int shared_base, int shared_rows,
                          int* counts, int* offsets, int* pos, int* pair, int* gu_list, int gu_bands, int gu_bands_shared,
                          int gu_slabs, int* dn_list, int dn_bands, int dn_slabs, int dn_slabs_shared, int kc_cap, int split,
                          int clear, int* done, int* err, cudaStream_t st);
int gemv_chunk_cap(int T);    // most K chunks per GEMV item at T tokens (sizes the partial-sum buffer)
constexpr int kGemvWarps = 4; // consumer warps of a GEMV CTA (one completion counter per item slot each)
int launch_gemv(bool gate_up, const GemvLaunch& L, cudaStream_t st);
int launch_seg_lists(const int* seg, int nseg, int shared_group, int shared_base, int shared_rows, int* gu_list,
                     int gu_bands, int gu_bands_shared, int* dn_list, int dn_bands, int bn, cudaStream_t st);
int launch_ep_regroup(const int* rc, int G, int El, const uint16_t* xrecv, int R, const uint16_t* xb, int t_real, int H,
                      int* seg, int* src_off, int* dst_off, uint16_t* xexp, int* rowmap, int* err, cudaStream_t st);
int launch_combine_y16(const float* res, const uint16_t* y, const int* pos, const int32_t* idx, const float* w,
                       const float* sgate, int shared_on, int T, int t_real, int k, int H, int P, float* out,
                       cudaStream_t st);
int launch_combine_bf16(float* out, const uint16_t* y, const int* pos, const int32_t* idx, const float* w, int T,
                        int t_real, int k, int H, cudaStream_t st);
// Peer-memory expert parallel (ep_peer.cu). sym[g] = rank g's symmetric buffer as mapped here.
constexpr int kMaxRanksPad = 64;   // ints per flag array in the symmetric buffer
struct EpPeerArgs {
    uint8_t* sym[kMaxRanks];
    size_t off_flags, off_cnt, off_meta, off_x, off_y;
    int* state;          // this rank's [0] epoch, [1] scatter blocks finished (in its symmetric buffer)
    int* err;            // the call's status words; err[1] != 0 stops every later exchange step
    int rank, G, E, El, H, k, r_cap;
    long long timeout_ns;
};
int launch_ep_post_counts(const EpPeerArgs& a, const int* counts, cudaStream_t st);
int launch_ep_plan_peer(const EpPeerArgs& a, int* send_base, int* seg, cudaStream_t st);
int launch_ep_scatter_rows(const EpPeerArgs& a, const uint16_t* xb, const int* pair, const int32_t* idx,
                           const int* offsets, const int* send_base, int P, int t_real, int sms, cudaStream_t st);
int launch_ep_wait(const EpPeerArgs& a, int which, cudaStream_t st);
int launch_ep_signal(const EpPeerArgs& a, int which, cudaStream_t st);
int launch_combine(const float* res, const float* y, const int* pos, const int32_t* idx, const float* w,
                   const float* sgate, int shared_on, int T, int t_real, int k, int H, int P, float* out, cudaStream_t st);


}  // namespace fm
