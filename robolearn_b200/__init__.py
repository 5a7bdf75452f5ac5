"""B200-native learner updates for RoboLearn-style FlashSAC and PPO.

Host code in Python calls hand-written sm_100a kernels in ``librl2.so`` through
a ctypes C ABI (``include/rl2.h``). PyTorch supplies device memory, streams,
CUDA graphs and ``torch.distributed``; there is no CPU or library fallback.
"""

__version__ = "0.1.0"
