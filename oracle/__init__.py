"""CPU restatement of the RoboLearn learner-update path — TEST INFRASTRUCTURE ONLY.

This package is the checker for the CUDA product path. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it. The product package ``robolearn_b200`` never imports it and has no CPU
fallback.

Pinning: ``flashsac_np`` is checked against golden tensors produced by running the
reference's own Torch FlashSAC (``src/robolearn/flashsac``) in this container
(``tests/golden/make_golden.py``). ``ppo_np`` is pinned by the known-answer tests of
``tests/test_warp_ppo.py`` in the reference and by golden tensors from a Torch
restatement of ``examples/diagnose_ppo_update.py:75-162`` (Warp itself is absent).
``philox_np`` restates the published Philox4x32-10 generator (Salmon et al., SC'11)
used by the device replay sampler; the reference's Warp RNG stream is unpinned and
replay parity is anchored on shared explicit indices, as the reference does
(``examples/diagnose_flash_replay.py:210-214``).
"""
