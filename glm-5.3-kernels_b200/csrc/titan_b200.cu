// Single translation unit of libtitan_b200.so: the launchers share the device
// error word defined in titan_abi.cu.
#include "titan_abi.cu"
#include "titan_kv.cu"
#include "titan_moe_align.cu"
#include "titan_moe_split_align.cu"
#include "titan_mla.cu"
#include "titan_index.cu"
#include "titan_io.cu"
#include "titan_moe_gemm.cu"
#include "titan_indexer.cu"
