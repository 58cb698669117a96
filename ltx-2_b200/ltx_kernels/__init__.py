"""B200-native (sm_100a) replacement of Lightricks/LTX-2's ``ltx_kernels`` blockwise-FP8 path.

Put the directory that contains this package (``ltx-2_b200/``) on ``sys.path``;
``ltx_kernels.blockwise`` then resolves to these kernels with the reference's
module names, op names and weight/scale layout.
"""
__version__ = "0.1.0"
