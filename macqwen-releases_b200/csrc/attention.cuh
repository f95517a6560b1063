// attention.cuh -- paged-KV decode attention (split-K flash decode).
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "../../include/fnmoe.h"

namespace fnmoe {

int paged_workspace_size(const FnPagedArgs *a, uint64_t *bytes, std::string &err);
int paged_decode(const FnPagedArgs *a, cudaStream_t s, std::string &err);

}  // namespace fnmoe
