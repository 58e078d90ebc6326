"""B200 (sm_100a) decode kernels behind the Python API of Charlie-Gzz/llm-decode-kernels.

Module map (same names as the reference's `kernels` package):
- `kernels.quant`      int4 pack/unpack, RTN quantizer, byte formula     (reference kernels/quant.py)
- `kernels.reference`  torch references used by the fp16 / w4_ref runner backends
- `kernels.w4a16`      W4A16 matmul                                       (reference kernels/w4a16.py)
- `kernels.fp8`        FP8 e4m3 weight-only matmul                        (reference kernels/fp8.py)
- `kernels.rmsnorm`    fused residual + RMSNorm                           (reference kernels/rmsnorm.py)
- `kernels.swiglu`     fused SwiGLU                                       (reference kernels/swiglu.py)
- `kernels.cuda.w4a16_cuda`  the M <= 16 decode entry point               (reference kernels/cuda/)
- `kernels.e2e`        Qwen2 runner with swappable backends, CUDA-graph decoder
- `kernels.bench`      CUDA-graph timing harness with rotating buffers

Every op runs a kernel of `lib/libdecodek.so` through its C ABI (include/decodek.h).
"""
