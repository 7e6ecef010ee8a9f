"""CPU checks of the drop-in boundary: the C-ABI library loads and exports every entry point the
header declares; the .gten writer produces images the oracle's reader (utils.cpp:29-61 order)
accepts; the device-free argument checks of the ABI return status codes."""
import os
import re
import subprocess

import numpy as np
import pytest

import gten_b200 as G
from gten_b200 import gtenfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gten_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(gtn_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = G.lib()
    names = declared_functions()
    assert len(names) >= 24
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", G.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (gtn_[a-z0-9_]+)", out))
    assert set(names) <= exported


def test_argument_errors_without_device():
    """Validation runs before any device work: bad descriptors give GTN_ERR_ARG (1)."""
    t = G.GT(0, G.Q8, (1, 32))  # NULL data pointer
    with pytest.raises(G.GtenError, match="status 1"):
        G.add(t, t, t)
    with pytest.raises(G.GtenError, match="status 1"):
        G.matmul_2d(G.GT(16, G.Q8, (1, 32)), G.GT(16, G.Q8, (4, 64)), G.GT(16, G.F32, (1, 4)))
    assert "matmul_2d" in G.lib().gtn_last_error().decode()


@pytest.mark.parametrize("kind,dims", [(6, [1000, 256, 2, 4, 2, 512, 0]), (6, [777, 192, 2, 3, 3, 320, 1]),
                                       (6, [900, 128, 3, 2, 2, 288, 2]), (3, None)])
@pytest.mark.parametrize("wdt", [G.Q8, G.Q4, G.F16])
def test_gten_image_roundtrip(orc, kind, dims, wdt):
    from oracle.oracle import OracleModel

    def pack(w, dt):
        return orc.pack_q8(w.numpy()) if dt == G.Q8 else orc.pack_q4(w.numpy())

    if kind == 3:  # OpenELM-sm: only check record sizes (the oracle loads it)
        img = gtenfile.synthetic_image(kind, wdt, 3, pack, std=0.02)
    else:
        img = gtenfile.synthetic_image(kind, wdt, 3, pack, dims=dims)
    OracleModel(orc, kind, wdt, 8, img, dims=dims)  # raises on any size mismatch
    bad = img.copy()
    bad[0] ^= 1
    with pytest.raises(ValueError):
        OracleModel(orc, kind, wdt, 8, bad, dims=dims)
    with pytest.raises(ValueError):
        OracleModel(orc, kind, wdt, 8, img[:-10], dims=dims)
