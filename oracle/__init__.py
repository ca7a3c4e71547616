"""CPU checkers for the batched NES env-step path (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of bench.py import this package.  The product
(``nesle_b200``) never does.

* :class:`Oracle` wraps ``liboracle.so`` -- the plain-C restatement of the
  reference kernel semantics (``nes_oracle.c``).
* :class:`Reference` wraps ``_ref/libnesle_ref.so`` -- the reference's own
  sources compiled unchanged (kind ``"B"``: batched headers on host vectors;
  kind ``"A"``: the ``nesle::Console`` CPU core).
"""
from .checker import Oracle, Reference, build, reference_available, FIELD_DTYPES

__all__ = ["Oracle", "Reference", "build", "reference_available", "FIELD_DTYPES"]
