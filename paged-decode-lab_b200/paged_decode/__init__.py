"""B200-native (sm_100a) paged split-K GQA decode attention.

Drop-in for ensigncode/paged-decode-lab's ``paged_decode`` package surface:
``runtime.DecodePlan``, ``workload.make_metadata`` / ``make_tensors`` and
``oracle.Layout``.  Importing this package never loads CUDA; the native library
is loaded when the first plan is built.
"""

__version__ = "0.1.0"
