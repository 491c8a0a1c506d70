"""CPU oracle for the diffucore_b200 hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
import this package, as the checker of the CUDA results or as the timed CPU restatement of the
reference's path. The product (``diffucore_b200``) never imports it.

``oracle/dc_oracle.c`` restates the reference's arithmetic (file:line in each function's
comment); it is pinned to the reference by the golden vectors under ``tests/golden/`` (made by
running the reference's own torch-op code) and, for the attention prep, by the reference's CUDA
prep kernels built from its source by ``oracle/build_ref.py`` into ``oracle/_ref/``.
``oracle/torch_ref.py`` restates the reference's torch-op (CPU) path of the W8A8 linear, pinned to
the reference's config-1 output hashes, and of each step of a FLUX block (``FluxOps``, pinned to
the reference's own FLUX output), and the reference's off-GPU ``Int8Linear`` forward as a module
(``CpuInt8Linear``, which makes this package's UNet reproduce the reference's); ``bench.py`` times
them as the CPU baselines of config 1, the FLUX step and the SDXL step.
"""

from .oracle import *  # noqa: F401,F403
