"""Tail-split choice of the attention grid (CPU: pure arithmetic exported by the extension).

The Wan2.1 480p shapes on a 148-SM B200: the 1-GPU step (12 heads, both CFG branches) fills its
last round well enough that no split pays; the per-rank shapes of CFG2 (12 heads), CFG2 x SP2
(6 heads) and CFG2 x SP4 (3 heads) cut their tail units into 2, 3 and 3 key ranges."""
import pytest

from ditserve_b200.ops._ext import available, ext

pytestmark = pytest.mark.skipif(not available(), reason="the sm_100a extension is not built in this tree")

S = 32760


@pytest.mark.parametrize("batch,heads,parts", [(2, 12, 1), (1, 12, 2), (1, 6, 3), (1, 3, 3)])
def test_wan_shapes(batch, heads, parts):
    assert ext().attention_tail_split_parts(batch, S, S, heads, 148) == parts


def test_no_split_when_rounds_are_full_or_keys_are_few():
    assert ext().attention_tail_split_parts(1, 256 * 148, 4096, 1, 148) == 1  # exactly one full round
    assert ext().attention_tail_split_parts(1, 4096, 1500, 3, 148) == 1       # 12 key tiles: no 8-tile ranges
    assert ext().attention_tail_split_parts(1, 4096, 4096, 3, 148) == 3       # 48 units: three ranges fill 144 SMs
