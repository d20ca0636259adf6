"""CPU parity checker for the rdv hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import anything from here. The
product (``rdv_project_b200``) never imports, links or executes this
package: every product call goes to the CUDA extension and fails loudly when
that extension is missing.

Contents

* ``c/oracle.c`` -> ``_build/liboracle.so``: row-by-row C restatement of the
  reference's Map arithmetic (Linear / LinearFast / ReLU chains), with
  float16/bfloat16 staging emulated through ``_Float16`` and bit tricks.
* ``ref_shim/`` -> ``_ref/libref_shaders.so``: the reference's OWN scalar
  GLSL functions (maps/linear.h, relu.h, composite.h,
  tensors/linear_tensor_op.h, relu_tensor_op.h, conv2d_tensor_op.h, the
  Winograd transforms of conv2d_tensor_op_winograd3x3.h and
  volumes/raymarching_transmittance_trait.h) compiled as C++ from the
  reference checkout. It pins the restatements below.
* ``mlp.py``, ``winograd.py``, ``raymarch.py``: numpy restatements; each
  function cites the reference file:line it follows.

Parity status: the fp32 Map/TensorOp paths, the Winograd transforms, the
filter transform and the fixed-step transmittance are pinned against the
reference's own code (golden fixtures in ``tests/golden``). The float16
cooperative-matrix GEMM, the pinhole camera (its GLSL uses array
constructors and ``out`` scalars that do not compile as C++) and the
emission-absorption compositing of BASELINE config 4 (not present in the
reference at all) are restatements: parity unpinned for those parts.
"""
