"""GPU test: building the networks is safe while another thread captures a
CUDA graph on the same device.

Group objects run on persistent worker threads; an object's networks are
built lazily by its first call, possibly while another object's worker on
the same GPU is capturing its refinement graph (thread-local capture mode).
Legacy-stream work or a device-wide synchronisation in that build fails with
"operation not permitted when stream is capturing" (seen with four objects
per GPU); the build now runs stream-ordered on a private stream. This test
holds a thread-local capture open on the main thread while a second thread
builds a network handle, then checks both succeed."""
from __future__ import annotations

import threading

import pytest

torch = pytest.importorskip("torch")

from fp_b200.kernels import FpkLibrary, Networks  # noqa: E402
from fp_b200.weights import make_default_packs  # noqa: E402

pytestmark = pytest.mark.gpu


def test_network_build_during_foreign_capture(tmp_path):
    refine, score = make_default_packs(tmp_path, seed=9)
    fpk = FpkLibrary()
    x = torch.zeros(1024, device="cuda")
    torch.cuda.synchronize()
    result = {}

    def build():
        try:
            for prec in (2, 3, 0):  # FP16, BF16 (device-side weight conversion), strict FP32
                nets = Networks(fpk, refine, score, prec, 2)
                nets.close()
            result["ok"] = True
        except Exception as e:  # noqa: BLE001 - reported through the assertion below
            result["error"] = str(e)

    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        g.capture_begin(capture_error_mode="thread_local")
        try:
            x.add_(1.0)
            t = threading.Thread(target=build)
            t.start()
            t.join(timeout=300)
            assert not t.is_alive()
        finally:
            g.capture_end()
    g.replay()
    torch.cuda.synchronize()
    assert result.get("ok"), result.get("error")
    assert x[0].item() == 1.0
