"""breeze_b200: B200-native (sm_100a) weight-only quantized decode linears.

Drop-in replacements for the reference's quantized linear modules and fused
decode kernels, backed by hand-written CUDA kernels in libbreeze_b200.so
(C ABI: include/breeze_b200.h):

  breeze_b200.int4_linear   Int4Linear, quantize_int4, quantize_module_int4
  breeze_b200.fp8_linear    Fp8Linear, quantize_module_fp8
  breeze_b200.int8_linear   Int8Linear, quantize_module_int8
  breeze_b200.fused.kernels FusedWeight, rms_gemv, rmsnorm, silu_mul

Put the ``breeze-tts-2_b200`` directory on sys.path to import it.
"""

__version__ = "0.1.0"
