// Single translation unit of libvq2_b200.so (keeps device globals and helpers in one module
// without relocatable device code).
#include "misc.cu"
#include "align.cu"
#include "decode.cu"
#include "prefill.cu"
#include "ep_p2p.cu"
#include "router.cu"
#include "pack.cu"
#include "shared.cu"
