// needle_b200: the whole library is this one translation unit, so that the
// device error word (nb::g_error_word) exists once per device and every
// kernel can name it directly.  Build: see needle_b200/build.py.
#include "nb_common.cuh"

#include "capi.cuh"
#include "kvcache.cuh"
#include "slots.cuh"
#include "decode.cuh"
#include "prefill.cuh"
#include "linear.cuh"
#include "norm.cuh"
#include "act.cuh"
#include "sample.cuh"
#include "swap.cuh"
#include "tp_allreduce.cuh"
#include "noalloc.cuh"
