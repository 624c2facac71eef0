// Allocation-free first-occurrence deduplication (C ABI).
//
// This entry point has no counterpart in the reference; it is an addition of
// this library for callers that cannot call cudaMalloc (a host program that
// owns all device memory through its own fixed pool, or a latency-critical
// call site that must not allocate).  Its working memory is a fixed ~9 MiB
// file-scope device array, which bounds one call to 262,144 keys; see
// unique_noalloc.cu for the full contract (return codes, first-call set-up
// before any stream capture, and the rule that overlapping calls race).
#pragma once

#include <cstdint>

#ifdef __cplusplus
extern "C" {
#endif

// keys: device int64[n]; unique, first_index: device int64[n]; inverse:
// device int32[n]; num_unique: device int32[1]; stream: cudaStream_t.
// Returns 0 on success, -1 if n > 262,144 (or negative), -2 if the scratch
// address could not be obtained, -3 if a launch failed.
int flare_unique_first_occurrence_noalloc(const int64_t* keys, int64_t n, int64_t* unique, int32_t* inverse,
                                          int64_t* first_index, int32_t* num_unique, void* stream);

// Forget the cached scratch address of `device`; call it after cudaDeviceReset on that device
// (the reset reloads the module, possibly at another address).  Returns 0, or -1 if out of range.
int flare_unique_noalloc_forget_device(int device);

#ifdef __cplusplus
}
#endif
