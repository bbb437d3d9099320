"""GPU: the TDT decoder's encoder projection (Decoder::project_encoder, decoder.rs:123-134) on the device against
the oracle's linear, bit for bit, for one frame (the reference's gemv order) and several (tile_rows order)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("t", [1, 2, 5, 37, 300])
def test_project_device_bit_exact(t):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import oracle
    from voxrt_b200 import synth
    from voxrt_b200._lib import check_device
    from voxrt_b200.decoder import TdtDecoder

    m = synth.decoder(seed=11)
    P = TdtDecoder(m, device=torch.cuda.current_device())
    O = oracle.TdtDecoder(m)
    enc = np.random.default_rng(t).standard_normal((t, m["d_model"])).astype(np.float32)
    got = P.project_device(torch.from_numpy(enc).cuda())
    torch.cuda.synchronize()
    check_device()
    want = O.project(enc)
    g = got.cpu().numpy()
    bad = np.flatnonzero(g.view(np.uint32) != want.view(np.uint32))
    assert bad.size == 0, f"{bad.size} mismatches, first {np.unravel_index(bad[0], g.shape)}"
