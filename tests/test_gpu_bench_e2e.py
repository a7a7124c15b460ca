"""GPU: the bench's end-to-end runner (pinned host buffers, row blocks on
three streams) returns exactly what one whole call of the candidate returns."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,shapes", [
    ("layer_norm", {"x": (1000, 2048), "weight": (2048,), "bias": (2048,)}),
    ("softmax", {"x": (37, 4096)}),
    ("sum_dim", {"x": (9, 100, 300)}),
    ("matmul", {"A": (500, 256), "B": (256, 384)}),
    ("diag_matmul", {"A": (300,), "B": (300, 128)}),
    ("mse_loss", {"predictions": (100000,), "targets": (100000,)}),  # not split: whole op
])
@pytest.mark.parametrize("chunks", [1, 4])
def test_e2e_runner_matches_whole_call(name, shapes, chunks, cuda_device):
    import bench
    from kbb200.workloads import WORKLOADS, make_inputs

    w = WORKLOADS[name]
    ins = make_inputs(w, cuda_device, seed=3, shapes=shapes)
    model = bench.load_candidate(w.problem).Model().to(cuda_device)
    with torch.no_grad():
        want = model(*ins).cpu()
    hin = [t.cpu().pin_memory() for t in ins]
    hout = torch.full(want.shape, float("nan"), dtype=want.dtype).pin_memory()
    streams = bench.E2EStreams(cuda_device)
    run = bench.e2e_runner(name, w.problem, hin, hout, cuda_device, chunks, streams)
    streams.begin()
    run()
    run()  # reuse of the device buffers while the first call may still run
    streams.end()
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(hout, want), name


@pytest.mark.parametrize("chunks", [1, 4])
def test_e2e_group_uploads_shared_input_once(chunks, cuda_device):
    """LayerNorm and RMSNorm of one x (the row-normalisation config): one
    upload per call feeds both forwards, and both results match whole calls."""
    import bench
    from kbb200.workloads import WORKLOADS, make_inputs

    w_ln, w_rms = WORKLOADS["layer_norm"], WORKLOADS["rms_norm"]
    ins = make_inputs(w_ln, cuda_device, seed=5, shapes={"x": (300, 2048), "weight": (2048,), "bias": (2048,)})
    ln = bench.load_candidate(w_ln.problem).Model().to(cuda_device)
    rms = bench.load_candidate(w_rms.problem).Model().to(cuda_device)
    with torch.no_grad():
        want_ln, want_rms = ln(*ins).cpu(), rms(*ins[:2]).cpu()
    hin = [t.cpu().pin_memory() for t in ins]
    h_ln = torch.full(want_ln.shape, float("nan")).pin_memory()
    h_rms = torch.full(want_rms.shape, float("nan")).pin_memory()
    streams = bench.E2EStreams(cuda_device)
    run = bench.e2e_runner("layer_norm", w_ln.problem, hin, h_ln, cuda_device, chunks, streams,
                           extra=[(rms, 2, h_rms)])
    streams.begin()
    run()
    run()
    streams.end()
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(h_ln, want_ln) and torch.equal(h_rms, want_rms)
