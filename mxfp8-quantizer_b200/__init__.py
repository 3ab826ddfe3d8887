"""B200-native MXFP8 quantizer: bf16/fp16 X -> E4M3 payload + UE8M0 scales in
the tcgen05 128x4 chunk layout.  The compute runs in libmxfp8.so (sm_100a
CUDA, C ABI in include/mxfp8.h); this package is the Python host side that
mirrors the reference's API (see quantizer.py)."""

from . import _capi, shard
from .quantizer import (
    DEFAULT_E2E_SUITE,
    DEFAULT_K_TILE,
    DEFAULT_ROWS_PER_CTA,
    FP8_E4M3_MAX,
    Q_BYTE_DIFF_TOLERANCE,
    SCALE_PACK_COLS,
    SCALE_ROWS_PER_PACK,
    SCALE_VEC_SIZE,
    CompiledQuantizer,
    HostQuantizer,
    MXFP8QuantizerConfig,
    blockscaled_gemm,
    build_runtime,
    check_cuda_launch_errors,
    decode_scale_bytes,
    dequantize,
    materialize_quantizer_buffers,
    pack_scale_bytes,
    packed_scale_storage_bytes,
    packed_scale_word_count,
    prepare_and_quantize,
    quantize,
    reference_quantize,
    run_e2e_suite,
    run_e2e_verification,
    run_quantizer,
    shape_problem,
    verify_quantizer_outputs,
)

__all__ = [n for n in dir() if not n.startswith("__")]
