// rows.cuh -- quantized embedding / n-gram row lookup.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "../../include/fnmoe.h"

namespace fnmoe {

int rows_dequant(const FnRowsArgs *a, cudaStream_t s, std::string &err);

}  // namespace fnmoe
