"""B200-native (sm_100a) INT8 hot path of DeepSeek-V3.2: act_quant, block-scaled int8_gemm,
lightning indexer + top-k, as drop-ins for hamzak-27/deepseek-v32-gtx1650's kernels.py API, plus
the producers either side of it (the indexer's Hadamard rotate + quantise, the weight block
quantiser) and the full indexer step with its int8 key cache.

The kernels live in libdsv32_int8.so (C ABI: include/dsv32_int8.h), built in-tree by
`python -m deepseek_v32_gtx1650_b200.build`.
"""
from .kernels import (GROUP, act_quant, int8_gemm, int8_gemm_partials, int8_index, int8_index_topk,
                      rotate_quant, select_topk, select_topk_parts, weight_quant)
from .kernels_v2 import (act_quant_kmajor, index_kmajor_k, index_kmajor_q, int8_gemm_v2, int8_index_v2, kmajor,
                         unkmajor)
from .hadamard_quant import fwht_quant_kmajor, hadamard_matrix, rotate_quant_kmajor, unpack_kmajor
from .indexer import KeyCache, indexer_step
from ._lib import Dsv32Error, device_status

__all__ = [
    "GROUP", "act_quant", "int8_gemm", "int8_gemm_partials", "int8_index", "int8_index_topk", "select_topk",
    "select_topk_parts",
    "act_quant_kmajor", "kmajor", "unkmajor", "int8_gemm_v2", "index_kmajor_q", "index_kmajor_k", "int8_index_v2",
    "rotate_quant", "weight_quant", "rotate_quant_kmajor", "fwht_quant_kmajor", "hadamard_matrix", "unpack_kmajor",
    "KeyCache", "indexer_step", "Dsv32Error", "device_status",
]
