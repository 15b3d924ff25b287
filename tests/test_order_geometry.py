"""The parameter-gradient order is fixed by the kernels' chunk geometry, and
the oracle restates it through constants of its own (oracle/canonical.py).
Bit-exact backward parity holds only while the two agree, so this checks
them against the constants in the CUDA sources, on the CPU."""
import re
from pathlib import Path

from oracle import canonical as C

CSRC = Path(__file__).resolve().parent.parent / "anima_flat_b200" / "csrc"


def _constexpr(name: str, path: Path) -> int:
    m = re.search(r"constexpr\s+int\s+" + name + r"\s*=\s*(\d+)\s*;", path.read_text())
    assert m, f"{name} not found in {path.name}"
    return int(m.group(1))


def test_adaln_bwd_chunk_matches_oracle():
    rows = _constexpr("kChunkRows", CSRC / "adaln_bwd.cu")
    assert C.BWD_WARPS * C.BWD_ROWS_PER_WARP == rows
    # the kernel's stages cut a chunk evenly
    assert rows % _constexpr("kStageRows", CSRC / "adaln_bwd.cu") == 0


def test_headnorm_bwd_chunk_matches_oracle():
    tokens = _constexpr("kHnbWarps", CSRC / "headnorm_bwd.cu")
    assert C.HN_WARPS * C.HN_TOK_PER_WARP == tokens
