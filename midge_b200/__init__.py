"""midge_b200 -- sm_100a-native quantized-MoE forward hot path of midge.

The product is the C-ABI library libmidgecuda.so (include/midgecuda.h) plus
the C host midge_b200/bin/midged; this package holds their sources, the
build script and a thin Python binding (abi.py) that the tests and the
bench drive.  Importing the package never touches the GPU; importing
midge_b200.abi loads the library and fails loudly if it is not built.
"""
__all__ = ["container"]
