"""The decode GEMM's synchronisation (csrc/gemm_decode_tc.cu) checked on a model
of its barrier protocol under random interleavings (tests/protocol_model.py):
for every CTA's unit range of the model's projection shapes and of the GPU
tests' shapes, no wait passes without its own phase completed and no state
deadlocks. The earlier issuer assignment (by position within a tile's segment)
is shown to fail, which is the race the kernel's assignment removes."""
import pytest

from protocol_model import cta_ranges, rule_by_segment, rule_by_unit, simulate

SHAPES = [(4096, 4096, 3), (4096, 4096, 1), (4096, 11008, 1), (11008, 4096, 1), (4096, 32000, 1),
          (128, 128, 1), (96, 256, 1), (1024, 640, 1), (11008, 512, 1), (2048, 1024, 1),
          (1001, 300, 1), (70, 132, 1), (4096, 256, 1), (1024, 512, 3), (11008, 128, 1)]


@pytest.mark.parametrize("k,n,batch", SHAPES)
def test_decode_gemm_protocol_has_no_race(k, n, batch):
    bad = []
    for nu, spt, u0 in cta_ranges(k, n, batch):
        for seed in (0, 1):
            errs = simulate(nu, spt, u0 % spt, rule=rule_by_unit, issuers=2, seed=seed)
            if errs:
                bad.append((u0, seed, errs[:2]))
    assert not bad, bad[:3]


def test_one_issuer_has_no_race():
    for nu, spt, u0 in cta_ranges(4096, 4096, 3):
        assert not simulate(nu, spt, u0 % spt, issuers=1, seed=0)


def test_segment_position_assignment_races():
    """Issuer by position in the segment: at a tile boundary an issuer can wait on
    a slot whose previous unit another issuer has not consumed yet, and the
    parity rule lets it pass on that earlier phase."""
    found = 0
    for nu, spt, u0 in cta_ranges(4096, 4096, 3):
        errs = simulate(nu, spt, u0 % spt, rule=rule_by_segment, issuers=2, seed=0)
        found += any("passed for completion" in e for e in errs)
    assert found > 0
