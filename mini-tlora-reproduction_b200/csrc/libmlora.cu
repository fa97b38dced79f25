// Single translation unit of the mlora native library (keeps device globals
// such as the error word visible to every kernel without relocatable device
// code).
#include "plan.cu"
#include "timing.cu"
#include "simt.cu"
#include "route.cu"
#include "tc.cu"
#include "allreduce.cu"
#include "multimem.cu"
#include "api.cu"
#include "noalloc.cu"
