"""B200 (sm_100a) block-scaled quantized GEMM: NVFP4 / MXFP8 / MXFP4 quantizers and
tcgen05 GEMM kernels behind the C ABI in include/qgemm.h."""
from .qgemm import (  # noqa: F401
    LAYOUT_MMA, LAYOUT_MMA_KMAJOR, LAYOUT_REF_LINEAR, Mxfp4Result, Mxfp8Result, Nvfp4Result,
    QGemmError, block_scaled_gemm, gemm_nvfp4_requant, lib, make_mxfp4, make_mxfp8, make_nvfp4,
    repack_nvfp4, sm1xx_scale_storage_size,
)
