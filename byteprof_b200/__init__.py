"""byteprof_b200: byteprof's decode hot path (skinny linear, fused mLSTM scan) on sm_100a kernels.

Operator API, mirroring the reference's modules (paths inside the byteprof project):
  byteprof_b200.optim.skinny        <- byteprof/optim/skinny.py          skinny_mm, dequantize
  byteprof_b200.optim.skinny_linear <- byteprof/optim/skinny_linear.py   SkinnyLinear
  byteprof_b200.quant.int8          <- byteprof/quant/triton_int8.py     gemv_int8, quantize_rowwise_int8
  byteprof_b200.quant.integrate     <- byteprof/quant/integrate.py       Int8Linear, apply_quantization
  byteprof_b200.quant.select        <- byteprof/quant/select.py          module selection rules
  byteprof_b200.optim.draft_fused   <- byteprof/optim/draft_fused.py     multistep_fw, lazy_commit, accept
  byteprof_b200.optim.draft_core    <- byteprof/optim/draft_core.py      mlstm_step_into (+ mlstm_scan)
The kernels live in one C-ABI library (include/bp_kernels.h) built by `byteprof_b200.build`.
"""

__version__ = "0.1.0"
