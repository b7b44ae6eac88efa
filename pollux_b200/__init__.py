"""pollux_b200 -- B200-native (sm_100a) implementation of the hot path of
alavicka/pollux: H24 nearest-codeword quantisation, 18-bit index pack/unpack
and LUT dequantisation, behind the reference's own Python signatures.

    import pollux_b200
    pollux_b200.install()      # route the reference modules' hot path here

Modules:
  castor         -- castor.py mirror (codebook, quantizer, pack/unpack, helpers)
  pack           -- pack._quantize_h24_layer and pack._quantize_int8 mirrors
  packed_linear  -- PackedH24Linear / PackedInt8* / materialize mirrors, batched materialize
  plx            -- .plx container reader / writer
  shard          -- row sharding across ranks, optional all-gather of packed bytes
  build          -- nvcc build recipe of libh24.so
"""
from __future__ import annotations

import sys

__version__ = "0.1.0"

# Names each reference module binds (directly or via `from castor import ...`)
# that this package replaces.
_PATCHES = {
    "castor": ["castor_quantize_leech", "pack_indices", "unpack_indices", "centers_to_indices",
               "CastorQuantizeLeech"],
    "pollux": ["castor_quantize_leech", "unpack_indices"],
    "pack": ["pack_indices", "_quantize_h24_layer", "_quantize_int8"],
}


def install(modules: dict | None = None) -> list[str]:
    """Rebind the hot-path functions of the reference's modules (castor,
    pollux, pack) to this package.  ``modules`` maps module names to module
    objects; by default the already-imported ``sys.modules`` entries are used.
    Returns the list of patched ``module.name`` strings."""
    from . import castor as c
    from . import pack as p
    from . import packed_linear as pl
    impl = {
        "castor_quantize_leech": c.castor_quantize_leech,
        "pack_indices": c.pack_indices,
        "unpack_indices": c.unpack_indices,
        "centers_to_indices": c.centers_to_indices,
        "CastorQuantizeLeech": c.CastorQuantizeLeech,
        "_quantize_h24_layer": p._quantize_h24_layer,
        "_quantize_int8": p._quantize_int8,
    }
    mods = modules if modules is not None else {k: sys.modules.get(k) for k in _PATCHES}
    done = []
    for modname, names in _PATCHES.items():
        mod = mods.get(modname)
        if mod is None:
            continue
        for name in names:
            if hasattr(mod, name):
                setattr(mod, name, impl[name])
                done.append(f"{modname}.{name}")
    pol = mods.get("pollux")
    if pol is not None and hasattr(pol, "PackedH24Linear"):
        pol.PackedH24Linear.materialize = pl.materialize
        done.append("pollux.PackedH24Linear.materialize")
    for cls in ("PackedInt8Embedding", "PackedInt8Linear"):
        if pol is not None and hasattr(pol, cls):
            getattr(pol, cls).materialize = pl.materialize_int8
            done.append(f"pollux.{cls}.materialize")
    return done
