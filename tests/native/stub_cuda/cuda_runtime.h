// Host-only stand-in for the CUDA runtime calls of leanstream_b200/csrc/ls_stream.cu
// (test infrastructure): lets the streaming engine's host logic -- admission
// order, reordering, READY words, completion callbacks, delays, retire -- be
// tested without a GPU. A "copy" is a memcpy that has landed by the time its
// event is queried.
#pragma once
#include <cstddef>
#include <cstring>

typedef int cudaError_t;
typedef struct StubStream* cudaStream_t;
typedef struct StubEvent {
    int recorded;
}* cudaEvent_t;
enum { cudaSuccess = 0, cudaErrorNotReady = 600 };
enum cudaMemcpyKind { cudaMemcpyHostToDevice = 1 };
#define cudaStreamNonBlocking 1
#define cudaEventDisableTiming 2

inline cudaError_t cudaGetDeviceCount(int* n) { *n = 1; return cudaSuccess; }
inline cudaError_t cudaGetDevice(int* d) { *d = 0; return cudaSuccess; }
inline cudaError_t cudaSetDevice(int) { return cudaSuccess; }
inline cudaError_t cudaStreamCreateWithFlags(cudaStream_t* s, unsigned) {
    *s = reinterpret_cast<cudaStream_t>(0x1);
    return cudaSuccess;
}
inline cudaError_t cudaStreamDestroy(cudaStream_t) { return cudaSuccess; }
inline cudaError_t cudaEventCreateWithFlags(cudaEvent_t* e, unsigned) {
    *e = new StubEvent{0};
    return cudaSuccess;
}
inline cudaError_t cudaEventDestroy(cudaEvent_t e) {
    delete e;
    return cudaSuccess;
}
inline cudaError_t cudaEventRecord(cudaEvent_t e, cudaStream_t) {
    e->recorded = 1;
    return cudaSuccess;
}
inline cudaError_t cudaEventQuery(cudaEvent_t) { return cudaSuccess; }
inline cudaError_t cudaMemcpyAsync(void* d, const void* s, size_t n, cudaMemcpyKind, cudaStream_t) {
    std::memcpy(d, s, n);
    return cudaSuccess;
}
