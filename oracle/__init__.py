"""TEST INFRASTRUCTURE — the CPU oracles for the MoE-FFN hot path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
package. It is the checker, never the thing measured or shipped.

Two oracles share one layer description (``oracle/moe_oracle.h``):

* ``Ref`` — the reference's own ggml-cpu implementation, compiled from the reference sources into
  ``oracle/_ref/`` (``make -C oracle ref``), driven by ``oracle/ref_runner.cpp`` ("O1").
* ``Port`` — this repository's plain-C restatement (``oracle/moe_oracle.c``), pinned against
  ``Ref`` and the golden fixtures under ``tests/golden/``.
"""
from .oracle import Port, Ref, LayerSpec, Sidecar, build_port, ref_available, port_available, sidecar_available  # noqa: F401
