// Implementation of tests/native/fake_cudart.h (see there).
#include "cuda_runtime_api.h"

#include <cstdlib>
#include <cstring>
#include <deque>
#include <string>
#include <vector>

struct FakeStream {
    int id;
};
struct FakeEvent {
    uint64_t seq = 0;     // copies that must be applied before the event completes
    bool recorded = false;
};

namespace {
struct Copy {
    char* to;
    const char* from;
    size_t width, height, to_pitch, from_pitch;
    std::vector<char> snapshot;   // source bytes captured at enqueue time
};
std::deque<Copy> queue;            // not yet applied
uint64_t enqueued = 0, applied = 0;
std::string failing;
int host_allocations = 0;
int host_registrations = 0;
uintptr_t last_stream = 0;

bool fail(const char* name) {
    if (failing == name) {
        failing.clear();
        return true;
    }
    return false;
}

void apply_until(uint64_t seq) {
    while (applied < seq && !queue.empty()) {
        Copy& c = queue.front();
        for (size_t r = 0; r < c.height; ++r)
            std::memcpy(c.to + r * c.to_pitch, c.snapshot.data() + r * c.width, c.width);
        queue.pop_front();
        ++applied;
    }
}

cudaError_t enqueue(void* to, size_t to_pitch, const void* from, size_t from_pitch, size_t width, size_t height,
                    cudaStream_t s) {
    Copy c{static_cast<char*>(to), static_cast<const char*>(from), width, height, to_pitch, from_pitch, {}};
    c.snapshot.resize(width * height);
    for (size_t r = 0; r < height; ++r)
        std::memcpy(c.snapshot.data() + r * width, static_cast<const char*>(from) + r * from_pitch, width);
    queue.push_back(std::move(c));
    ++enqueued;
    last_stream = reinterpret_cast<uintptr_t>(s);
    return cudaSuccess;
}
}  // namespace

extern "C" {
const char* cudaGetErrorString(cudaError_t rc) { return rc == cudaErrorNotReady ? "not ready" : "injected CUDA error"; }
cudaError_t cudaSetDevice(int) { return fail("cudaSetDevice") ? cudaErrorInjected : cudaSuccess; }
cudaError_t cudaHostAlloc(void** p, size_t size, unsigned) {
    if (fail("cudaHostAlloc")) return cudaErrorInjected;
    *p = std::calloc(1, size);
    if (!*p) return cudaErrorInjected;
    ++host_allocations;
    return cudaSuccess;
}
cudaError_t cudaFreeHost(void* p) {
    std::free(p);
    --host_allocations;
    return cudaSuccess;
}
cudaError_t cudaStreamCreateWithFlags(cudaStream_t* s, unsigned) {
    static int next = 1;
    *s = new FakeStream{next++};
    return cudaSuccess;
}
cudaError_t cudaStreamSynchronize(cudaStream_t) {
    if (fail("cudaStreamSynchronize")) return cudaErrorInjected;
    apply_until(enqueued);
    return cudaSuccess;
}
cudaError_t cudaDeviceSynchronize(void) {
    if (fail("cudaDeviceSynchronize")) return cudaErrorInjected;
    apply_until(enqueued);
    return cudaSuccess;
}
cudaError_t cudaStreamQuery(cudaStream_t) { return queue.empty() ? cudaSuccess : cudaErrorNotReady; }
cudaError_t cudaStreamDestroy(cudaStream_t s) {
    delete s;
    return cudaSuccess;
}
cudaError_t cudaStreamWaitEvent(cudaStream_t, cudaEvent_t, unsigned) {
    return fail("cudaStreamWaitEvent") ? cudaErrorInjected : cudaSuccess;
}
cudaError_t cudaEventCreateWithFlags(cudaEvent_t* e, unsigned) {
    if (fail("cudaEventCreateWithFlags")) return cudaErrorInjected;
    *e = new FakeEvent();
    return cudaSuccess;
}
cudaError_t cudaEventRecord(cudaEvent_t e, cudaStream_t) {
    if (fail("cudaEventRecord")) return cudaErrorInjected;
    e->seq = enqueued;
    e->recorded = true;
    return cudaSuccess;
}
cudaError_t cudaEventSynchronize(cudaEvent_t e) {
    if (fail("cudaEventSynchronize")) return cudaErrorInjected;
    if (e->recorded) apply_until(e->seq);
    return cudaSuccess;
}
cudaError_t cudaEventQuery(cudaEvent_t e) { return !e->recorded || applied >= e->seq ? cudaSuccess : cudaErrorNotReady; }
cudaError_t cudaEventDestroy(cudaEvent_t e) {
    delete e;
    return cudaSuccess;
}
cudaError_t cudaMemcpyAsync(void* to, const void* from, size_t size, cudaMemcpyKind, cudaStream_t s) {
    if (fail("cudaMemcpyAsync")) return cudaErrorInjected;
    return enqueue(to, size, from, size, size, 1, s);
}
cudaError_t cudaMemcpy2DAsync(void* to, size_t to_pitch, const void* from, size_t from_pitch, size_t width,
                              size_t height, cudaMemcpyKind, cudaStream_t s) {
    if (fail("cudaMemcpy2DAsync")) return cudaErrorInjected;
    return enqueue(to, to_pitch, from, from_pitch, width, height, s);
}

void fake_cuda_fail_next(const char* call) { failing = call; }
int fake_cuda_pending(void) { return int(queue.size()); }
int fake_cuda_live_host_allocations(void) { return host_allocations; }
uintptr_t fake_cuda_last_stream(void) { return last_stream; }
void fake_cuda_discard_pending(void) {
    applied += queue.size();
    queue.clear();
}
}

extern "C" cudaError_t cudaHostRegister(void* ptr, size_t size, unsigned) {
    if (fail("cudaHostRegister")) return cudaErrorInjected;
    if (!ptr || !size) return cudaErrorInjected;
    ++host_registrations;
    return cudaSuccess;
}

extern "C" cudaError_t cudaHostUnregister(void* ptr) {
    if (fail("cudaHostUnregister")) return cudaErrorInjected;
    if (!ptr) return cudaErrorInjected;
    --host_registrations;
    return cudaSuccess;
}

extern "C" int fake_cuda_live_host_registrations(void) { return host_registrations; }

extern "C" cudaError_t cudaGetLastError(void) { return cudaSuccess; }
