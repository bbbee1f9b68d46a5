"""Device side of the on-disk table format: a CUDA table (float16 values,
float32 accumulators) saved through pinned chunks and reloaded onto the GPU
at another world size."""

import numpy as np
import pytest
import torch

from model_b200 import table_io

pytestmark = pytest.mark.gpu


def test_device_round_trip_small_chunks(tmp_path, monkeypatch):
    monkeypatch.setattr(table_io, "_CHUNK_BYTES", 4096)       # many chunks through the pinned buffer
    n, d = 5000, 64
    g = torch.Generator("cuda").manual_seed(0)
    full_v = torch.randn(n, d, device="cuda", generator=g).half()
    full_a = torch.rand(n, device="cuda", generator=g)
    # the reference layout of the whole table, then its rows at world 2 on the device
    table_io.save_table(str(tmp_path / "all"), {"values": full_v, "acc": full_a}, n)
    np.testing.assert_array_equal(np.load(tmp_path / "all" / "values.npy"), full_v.cpu().numpy())
    for r in range(2):
        got = table_io.load_table(str(tmp_path / "all"), ["values", "acc"], rank=r, world=2,
                                  device=torch.device("cuda"))
        assert got["values"].is_cuda and got["values"].dtype == torch.float16
        assert torch.equal(got["values"], full_v[r::2])
        assert torch.equal(got["acc"], full_a[r::2])
