// The inline-PTX building blocks live in the public device headers, where the
// kernels that environment translation units instantiate can reach them.
#pragma once

#include "metalgym/detail/ptx.cuh"
