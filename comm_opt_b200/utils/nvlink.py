"""NVLink traffic of one GPU from NVML's cumulative throughput counters (read-only).

The reference measured NVLink RX/TX utilisation with nsys GPU metrics around NVTX ranges
(exp/M11_before_prototype/run.py:38-40); nsys is not part of this stack. NVML keeps per-link counters of
the data bytes sent and received over NVLink (NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX / _RX, KiB, scope =
link index); reading them before and after a run gives the bytes that crossed this GPU's links, e.g. to
check that a one-shot all-reduce of S bytes on W ranks sends (W - 1) x S per rank, and to put a measured
byte count into a roofline instead of a formula. Nothing here changes a GPU setting.

    ctr = NvlinkCounters(device_index=0)
    with ctr.measure() as m:
        ...  # the work; synchronize before leaving the block
    print(m["tx_bytes"], m["rx_bytes"])

The counters are sampled by the driver, so short runs should be repeated until the delta is large
(hundreds of MB) against the counter granularity.
"""
from __future__ import annotations

import contextlib
import time


class NvlinkCounters:
    def __init__(self, device_index: int = 0, nvml=None):
        if nvml is None:
            import pynvml as nvml
        self.nvml = nvml
        nvml.nvmlInit()
        self.handle = nvml.nvmlDeviceGetHandleByIndex(device_index)
        self.links = self._active_links()
        self.fields = (nvml.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX, nvml.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_RX)

    def _active_links(self) -> list[int]:
        nv = self.nvml
        out = []
        for link in range(getattr(nv, "NVML_NVLINK_MAX_LINKS", 18)):
            try:
                if nv.nvmlDeviceGetNvLinkState(self.handle, link) == nv.NVML_FEATURE_ENABLED:
                    out.append(link)
            except nv.NVMLError:
                continue  # link not present on this part
        return out

    @property
    def available(self) -> bool:
        return bool(self.links)

    def read(self) -> dict:
        """Cumulative KiB sent / received over all active links (links whose counter read failed are
        listed in `failed_links`)."""
        req = [(f, link) for link in self.links for f in self.fields]
        vals = self.nvml.nvmlDeviceGetFieldValues(self.handle, req) if req else []
        tx = rx = 0
        failed = set()
        for (f, link), v in zip(req, vals):
            if v.nvmlReturn != 0:
                failed.add(link)
                continue
            if f == self.fields[0]:
                tx += int(v.value.ullVal)
            else:
                rx += int(v.value.ullVal)
        return dict(tx_kib=tx, rx_kib=rx, failed_links=sorted(failed))

    @contextlib.contextmanager
    def measure(self, settle_s: float = 0.1):
        """Yields a dict that holds tx_bytes / rx_bytes of the block when it exits; waits settle_s before the
        final read so that the driver's sampled counters include the end of the block."""
        out: dict = {}
        a = self.read()
        try:
            yield out
        finally:
            if settle_s > 0:
                time.sleep(settle_s)
            b = self.read()
            out.update(tx_bytes=(b["tx_kib"] - a["tx_kib"]) * 1024, rx_bytes=(b["rx_kib"] - a["rx_kib"]) * 1024,
                       links=len(self.links), failed_links=sorted(set(a["failed_links"]) | set(b["failed_links"])))
