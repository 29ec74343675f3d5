"""A fake of pynvml's interface for CPU tests: an 8-GPU NVSwitch box whose links,
P2P status, persistence and processes a test can change."""

from types import SimpleNamespace


class FakeNVML:
    NVML_NVLINK_MAX_LINKS = 18
    NVML_FEATURE_ENABLED = 1
    NVML_FEATURE_DISABLED = 0
    NVML_P2P_CAPS_INDEX_NVLINK = 3
    NVML_P2P_STATUS_OK = 0
    NVML_COMPUTEMODE_DEFAULT = 0
    NVML_MEMORY_ERROR_TYPE_UNCORRECTED = 1
    NVML_VOLATILE_ECC = 0

    PCI = ["0000:1b:00.0", "0000:43:00.0", "0000:52:00.0", "0000:61:00.0", "0000:9d:00.0", "0000:c3:00.0",
           "0000:d1:00.0", "0000:df:00.0"]

    def __init__(self, n=8):
        self.n = n
        self.links = {i: 18 for i in range(n)}
        self.p2p_broken = set()
        self.persistence = {i: 1 for i in range(n)}
        self.procs = {i: [] for i in range(n)}
        self.ecc = {i: 0 for i in range(n)}
        self.tx = {i: 0 for i in range(n)}
        self.errors = {i: 0 for i in range(n)}

    def nvmlInit(self):
        pass

    def nvmlDeviceGetCount(self):
        return self.n

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetName(self, h):
        return b"NVIDIA B200"

    def nvmlDeviceGetUUID(self, h):
        return f"GPU-{h:08x}-0000-4000-8000-{h:012x}"

    def nvmlDeviceGetPciInfo(self, h):
        return SimpleNamespace(busId=("0000" + self.PCI[h]).encode())

    def nvmlDeviceGetNumaNodeId(self, h):
        return 0 if h < 4 else 1

    def nvmlDeviceGetNvLinkState(self, h, link):
        if link >= 18:
            raise RuntimeError("no such link")
        return 1 if link < self.links[h] else 0

    def nvmlDeviceGetNvLinkRemotePciInfo_v2(self, h, link):
        return SimpleNamespace(busId=f"00000000:{0xa0 + link % 4:02x}:00.0".encode())  # NVSwitch functions

    def nvmlDeviceGetP2PStatus(self, a, b, index):
        return 1 if (min(a, b), max(a, b)) in self.p2p_broken else 0

    def nvmlDeviceGetPersistenceMode(self, h):
        return self.persistence[h]

    def nvmlDeviceGetComputeMode(self, h):
        return 0

    def nvmlDeviceGetTotalEccErrors(self, h, kind, counter):
        return self.ecc[h]

    def nvmlDeviceGetComputeRunningProcesses(self, h):
        return self.procs[h]

    def nvmlSystemGetDriverVersion(self):
        return "580.159"

    def nvmlSystemGetCudaDriverVersion(self):
        return 13000

    def nvmlDeviceGetFieldValues(self, h, ids):
        out = []
        for fid in ids:
            out.append(SimpleNamespace(nvmlReturn=0, value=SimpleNamespace(ullVal=self.tx[h] + fid)))
        return out

    def nvmlDeviceGetNvLinkErrorCounter(self, h, link, code):
        if link >= 18:
            raise RuntimeError("no such link")
        return self.errors[h] if link == 0 else 0
