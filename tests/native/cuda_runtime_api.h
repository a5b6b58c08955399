// Test-only: routes the pool's <cuda_runtime_api.h> to the fake runtime.
#pragma once
#include "fake_cudart.h"
