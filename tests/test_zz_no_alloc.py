"""tb_frontend_static: the front-end for callers that cannot allocate device memory
(a real-time audio thread, where cudaMalloc can synchronize the device and stall the
stream; a host whose device memory belongs to another allocator). It keeps its scratch in
a fixed array inside the library instead of a caller-supplied workspace; its features
must equal tb_frontend's, call after call, since the array keeps the previous call's
contents; the same kernels run on the same inputs, so bit for bit. Collected last, so a run that stops at the first failure has run the rest."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def front_end_model(L, keep):
    """A tb_model with only the front-end tables set (window and sparse mel filters)."""
    from tinybark_b200 import tables

    mel_w, mel_start, mel_off = tables.sparse_mel()
    arrays = [torch.from_numpy(a).cuda() for a in (tables.window(), mel_w, mel_start, mel_off)]
    keep.extend(arrays)
    m = L.Model()
    m.window, m.mel_w, m.mel_start, m.mel_off = (a.data_ptr() for a in arrays)
    return m


def packed(clips):
    sizes = np.array([len(c) for c in clips], np.int64)
    soff = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    frames = sizes // 160
    foff = np.concatenate([[0], np.cumsum(frames)]).astype(np.int32)
    return (torch.from_numpy(np.concatenate(clips)).cuda(), torch.from_numpy(soff).cuda(),
            torch.from_numpy(foff).cuda(), int(foff[-1]))


def test_static_front_end_matches_workspace_front_end_twice():
    from tinybark_b200 import _lib as L
    from tinybark_b200 import synthetic

    torch.cuda.set_device(0)
    keep = []
    model = front_end_model(L, keep)
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(4)
    full = [synthetic.to_float(synthetic.clip(float(s), 200 + i))
            for i, s in enumerate(rng.uniform(0.02, 12.0, L.FRONTEND_STATIC_MAX_CLIPS))]
    batches = [
        [synthetic.to_float(synthetic.clip(s, 70 + i)) for i, s in enumerate((3.1, 0.02, 12.0, 7.77, 1.0))],
        [synthetic.to_float(synthetic.clip(s, 90 + i)) for i, s in enumerate((0.5, 29.9, 2.2))],
        full,  # exactly as many clips as the scratch holds
        full[:2],
    ]
    for clips in batches:
        samples, soff, foff, frames = packed(clips)
        ref = torch.empty(frames, 128, device="cuda")
        nbytes = L.lib.tb_frontend_workspace_bytes(len(clips), frames)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        L.check(L.lib.tb_frontend(ctypes.byref(model), samples.data_ptr(), soff.data_ptr(), foff.data_ptr(),
                                  len(clips), frames, 0, ref.data_ptr(), ws.data_ptr(), nbytes, stream), "tb_frontend")
        got = torch.full((frames, 128), float("nan"), device="cuda")
        L.check(L.lib.tb_frontend_static(ctypes.byref(model), samples.data_ptr(), soff.data_ptr(), foff.data_ptr(),
                                         len(clips), frames, got.data_ptr(), stream), "tb_frontend_static")
        torch.cuda.synchronize()
        # The same kernels on the same inputs: the same bits.
        np.testing.assert_array_equal(got.cpu().numpy(), ref.cpu().numpy())


def test_static_front_end_rejects_batches_beyond_its_scratch():
    from tinybark_b200 import _lib as L

    keep = []
    model = front_end_model(L, keep)
    n = L.FRONTEND_STATIC_MAX_CLIPS + 1
    samples = torch.zeros(n * 320, device="cuda")
    soff = torch.arange(0, (n + 1) * 320, 320, dtype=torch.int64, device="cuda")
    foff = torch.arange(0, (n + 1) * 2, 2, dtype=torch.int32, device="cuda")
    out = torch.empty(n * 2, 128, device="cuda")
    status = L.lib.tb_frontend_static(ctypes.byref(model), samples.data_ptr(), soff.data_ptr(), foff.data_ptr(), n,
                                      2 * n, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert status == 5
    with pytest.raises(RuntimeError, match="scratch"):
        L.check(status, "tb_frontend_static")
