// sosob200.cu -- the whole device library as one translation unit (so the
// device-side globals in common.cuh have exactly one definition).
#include "common.cuh"
#include "matvec.cuh"
#include "norm.cuh"
#include "decode_ops.cuh"
#include "mla.cuh"
#include "dispatch.cuh"
#include "engine.cuh"
#include "noalloc.cuh"
#include "prefill.cuh"
#include "block.cuh"
#include "prefill_engine.cuh"
#include "som.cuh"
