"""pyre_b200: B200-native (sm_100a) tensor-parallel forward hot path of Pyre.

Host code is Python over PyTorch device tensors; the arithmetic is hand-written CUDA in
``libpyre_b200.so`` behind the C ABI of ``include/pyre_b200.h``. There is no CPU path.
"""
__version__ = "0.1.0"
