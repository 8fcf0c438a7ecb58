"""B200-native FlashGRPO speculative rollout step (MEDUSA tree verify).

Drop-in for the reference's ``flashgrpo_b200`` rollout path: the same module
layout (``decoding``, ``models``) and public names, with the hot path running
as sm_100a CUDA kernels behind the C ABI declared in ``include/fg_b200.h``.
"""

__version__ = "0.1.0"
