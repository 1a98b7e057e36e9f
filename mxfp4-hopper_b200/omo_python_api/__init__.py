"""The reference's Python operator API (code/kernel/api/), served by the B200 `omo`.

`omo_python_api.mxfp4` and `omo_python_api.mxfp4_dequant` keep the reference's
function names, arguments, output allocation, padding and splitting, so the
Transformer Engine and Megatron patches that import them run unchanged.
"""
import mxfp4_b200  # noqa: F401  (puts the package directory, home of `omo`, on sys.path)
