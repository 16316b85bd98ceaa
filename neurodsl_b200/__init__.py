"""NeuroDSL B200: the transformer-inference hot path of NeuroDSL on sm_100a.

The compute lives in ``libneurodsl_b200.so`` (C ABI, ``include/neurodsl_b200.h``);
``neurodsl_b200.ops`` calls it on torch CUDA tensors and
``neurodsl_b200.graph`` mirrors NeuroDSL's GraphRule / register_op! / demand!
operator API on top of it.
"""
__version__ = "0.1.0"
