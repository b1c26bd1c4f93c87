// C entry point over the reference's own host router (TEST INFRASTRUCTURE ONLY).
//
// Compiled by oracle/Makefile together with the reference source
// src/open_qwen36/block_host.cpp (read in place, never copied) into oracle/_ref/libref_router.so.
// Only tests/ and bench.py's CPU-baseline leg load it: it validates the oracle restatement and is
// the timed "reference" CPU baseline of the router stage (block_host.cpp:766-803, OpenMP).
#include <cstddef>
#include <cstdint>
#include <exception>

namespace open_qwen36 {
namespace host {
void router_block(size_t T, size_t hid, size_t E, size_t topk, const float* xm, const float* Wr, float* probs,
                  int32_t* idx, float* w);
}
}  // namespace open_qwen36

extern "C" int ref_router_block(size_t T, size_t hid, size_t E, size_t topk, const float* xm, const float* Wr,
                                float* probs, int32_t* idx, float* w) {
    try {
        open_qwen36::host::router_block(T, hid, E, topk, xm, Wr, probs, idx, w);
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}
