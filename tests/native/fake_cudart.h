// A stand-in CUDA runtime API for testing the pinned pool's control flow on a
// CPU. Host malloc plays pinned memory; async copies are queued and applied only
// when a synchronize reaches them, so "in flight" is observable; any call can
// be made to fail once. It proves error handling, never CUDA behaviour.
#pragma once
#include <cstddef>
#include <cstdint>

typedef int cudaError_t;
typedef struct FakeStream* cudaStream_t;
typedef struct FakeEvent* cudaEvent_t;

enum : int { cudaSuccess = 0, cudaErrorNotReady = 600, cudaErrorInjected = 999 };
enum : unsigned { cudaHostAllocPortable = 1, cudaHostAllocMapped = 2, cudaStreamNonBlocking = 1,
                  cudaEventDisableTiming = 2, cudaHostRegisterPortable = 1, cudaHostRegisterMapped = 2,
                  cudaHostRegisterReadOnly = 8 };
enum cudaMemcpyKind { cudaMemcpyHostToDevice = 1, cudaMemcpyDeviceToHost = 2 };

extern "C" {
const char* cudaGetErrorString(cudaError_t);
cudaError_t cudaSetDevice(int);
cudaError_t cudaHostAlloc(void**, size_t, unsigned);
cudaError_t cudaFreeHost(void*);
cudaError_t cudaHostRegister(void*, size_t, unsigned);
cudaError_t cudaHostUnregister(void*);
cudaError_t cudaGetLastError(void);
cudaError_t cudaStreamCreateWithFlags(cudaStream_t*, unsigned);
cudaError_t cudaStreamSynchronize(cudaStream_t);
cudaError_t cudaDeviceSynchronize(void);
cudaError_t cudaStreamQuery(cudaStream_t);
cudaError_t cudaStreamDestroy(cudaStream_t);
cudaError_t cudaStreamWaitEvent(cudaStream_t, cudaEvent_t, unsigned);
cudaError_t cudaEventCreateWithFlags(cudaEvent_t*, unsigned);
cudaError_t cudaEventRecord(cudaEvent_t, cudaStream_t);
cudaError_t cudaEventSynchronize(cudaEvent_t);
cudaError_t cudaEventQuery(cudaEvent_t);
cudaError_t cudaEventDestroy(cudaEvent_t);
cudaError_t cudaMemcpyAsync(void*, const void*, size_t, cudaMemcpyKind, cudaStream_t);
cudaError_t cudaMemcpy2DAsync(void*, size_t, const void*, size_t, size_t, size_t, cudaMemcpyKind, cudaStream_t);

// Test controls.
void fake_cuda_fail_next(const char* call);   // the next call of that name returns cudaErrorInjected
int fake_cuda_pending(void);                   // queued copies not yet applied
int fake_cuda_live_host_allocations(void);     // cudaHostAlloc minus cudaFreeHost
int fake_cuda_live_host_registrations(void);   // cudaHostRegister minus cudaHostUnregister
uintptr_t fake_cuda_last_stream(void);         // stream of the last queued copy
void fake_cuda_discard_pending(void);          // drop queued copies without applying them
}
