// Single translation unit of libcpde_b200.so: the engine and its C ABI.
#include "engine.cu"
#include "capi.cu"
#include "noalloc.cu"
