"""Index build on the GPU (``SeoulKV4Index.build(..., build_device="cuda")``).

The clustering, the CSR lists and the group-scale centroid codec run on the
device.  The codec is checked byte for byte against the reference's own
output (the golden fixture) and against the host codec on a full-size cell;
a CUDA-built index passes the structural checks and decodes like the oracle.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from seoulkv_b200 import SeoulKV4, SeoulKV4Config, SeoulKV4Index, _clustering, _codecs, synthetic
from tests.helpers import Case, Golden, bits

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3
FIELDS = ("upper", "lower", "scale", "group_fine_scale", "fine_scale", "coarse_residual_norm", "coarse2",
          "offsets", "values", "levels", "centroids", "decoded", "coarse_odd", "coarse_centroids")


def _raw(t):
    return (t.view(torch.int16) if t.dtype in (torch.float16, torch.bfloat16) else t).numpy()


def test_device_codec_matches_reference_fixture(cuda):
    """The codec on CUDA tensors gives the reference's bytes (fixture from its own encoder)."""
    z = Golden().z
    cell = dict(centroids=torch.from_numpy(z["codec_in_centroids"].copy()).view(torch.float16).to(cuda),
                offsets=torch.from_numpy(z["codec_in_offsets"].copy()).to(cuda),
                values=torch.from_numpy(z["codec_in_values"].copy()).to(cuda))
    enc = _codecs.encode_group_scale_cell(cell)
    for name in FIELDS:
        assert enc[name].device.type == "cpu", name
        assert np.array_equal(_raw(enc[name]), z[f"codec_out_{name}"]), name


def test_device_codec_matches_host_at_full_size(cuda):
    """A 128K-context cell (nc = 32,672): device and host codecs agree byte for byte."""
    nc, tokens = 32672, 130688
    g = torch.Generator().manual_seed(7)
    cent = _clustering.midrise4(torch.randn(nc, 256, generator=g) * torch.rand(nc, 1, generator=g)).half()
    labels = torch.stack([torch.randint(0, nc, (tokens,), generator=g), torch.randint(0, nc, (tokens,), generator=g)], 1)
    labels[:, 1] = torch.where(labels[:, 1] == labels[:, 0], (labels[:, 0] + 1) % nc, labels[:, 1])
    off_h, val_h = _clustering.to_csr(labels, nc)
    off_d, val_d = _clustering.to_csr(labels.to(cuda), nc)
    assert np.array_equal(off_h.numpy(), off_d.cpu().numpy()) and np.array_equal(val_h.numpy(), val_d.cpu().numpy())
    host = _codecs.encode_group_scale_cell(dict(centroids=cent, offsets=off_h, values=val_h))
    dev = _codecs.encode_group_scale_cell(dict(centroids=cent.to(cuda), offsets=off_d, values=val_d))
    for name in FIELDS:
        assert np.array_equal(_raw(host[name]), _raw(dev[name])), name


def test_cuda_built_index_decodes_like_the_oracle(cuda):
    """build_device="cuda": structurally valid cells; ids bit-exact and output in tolerance."""
    context, seed = 16384, 41
    k, v, _ = synthetic.make_kv(context, seed=seed, components=256)
    index = SeoulKV4Index.build(k, v, sink=128, local=256, nprobe=128, build_device=cuda)
    for c in index.cells():
        _codecs.validate_static_cell(c)
        _codecs.require_group_scale_cell(c)
    case = Case(context=context, seed=seed, index=index)
    with SeoulKV4(device=cuda, k=case.k, v=case.v, index=index, config=SeoulKV4Config(debug=True)) as attn:
        for qs in (3, 4):
            q = case.query(qs)
            y = attn.run(q).to_torch()
            ids = attn.debug_snapshot()["selected_ids"].numpy()
            res, ref = case.oracle(q)
            assert np.array_equal(ids, np.stack([r["final_ids"] for r in res])), f"query {qs}: ids"
            err = np.abs(O.bf16_to_f32(bits(y).reshape(16, 256)).astype(np.float64)
                         - O.bf16_to_f32(ref).astype(np.float64))
            assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())
