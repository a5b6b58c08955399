// Internal helpers shared by the translation units of _cuda_native.so.
#pragma once

// Set the calling thread's kvsnap_cuda_error() text.
void kvsnap_internal_set_error(const char* message);
