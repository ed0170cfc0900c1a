"""The memory-bound kernel sweep: achieved HBM bandwidth of every memory-bound
kernel the encoder plan dispatches, over rows 4K-4M x widths {64, 768, 1024,
4096} (transposes: T up to 65536, H 12 and 16, D 64), as a fraction of the
device's measured copy bandwidth.

Bytes are the kernel's ALGORITHMIC traffic -- one read of every input and one
write of every output at storage width -- so a kernel that re-reads its input
does not get credit for it:

    softmax, scale, transpose_th, transpose_hd   4 B per element
    rope_2d    4 B per element + the T x D fp32 cos and sin tables
    add        6 B per element (two fp16 reads, one fp16 write)
    cast       6 B per element (fp32 read, fp16 write)
    layernorm  4 B per element + 2 C fp32 parameters
    rmsnorm    4 B per element + C fp16 gains

Each case is timed with CUDA events around single launches on the current
stream, after warm-up, with a 256 MiB L2 flush between launches (outside the
timed pairs) so small cases are not served from the 126 MB L2. Cases whose
tensors would exceed `max_tensor_bytes` or 2^31 elements are skipped. Small
cases are launch-latency bound and say so through their low fraction.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from hexlib_b200 import _lib

ROWS = (4096, 65536, 1 << 20, 4 << 20)
WIDTHS = (64, 768, 1024, 4096)
TRANSPOSE_T = (4096, 16384, 65536)
TRANSPOSE_H = (12, 16)
D_HEAD = 64
KINDS = ("softmax", "layernorm", "rmsnorm", "rope_2d", "add", "scale", "cast",
         "transpose_th", "transpose_hd")


@dataclass(frozen=True)
class Case:
    kind: str
    rows: int          # R (row kernels), T (rope, transposes), M (matmul_epilogue)
    width: int         # C (row kernels), H*D (rope, transposes), N (matmul_epilogue)
    heads: int = 0     # H for rope and the transposes
    depth: int = 0     # K (matmul_epilogue; its epilogue is bias + gelu_tanh)

    @property
    def flops(self) -> int:
        return 2 * self.rows * self.width * self.depth if self.kind == "matmul_epilogue" else 0

    @property
    def elems(self) -> int:
        return self.rows * self.width

    @property
    def bytes(self) -> int:
        e = self.elems
        if self.kind in ("softmax", "scale", "transpose_th", "transpose_hd"):
            return 4 * e
        if self.kind == "rope_2d":
            return 4 * e + 2 * self.rows * D_HEAD * 4
        if self.kind in ("add", "cast"):
            return 6 * e
        if self.kind == "layernorm":
            return 4 * e + 2 * self.width * 4
        if self.kind == "rmsnorm":
            return 4 * e + 2 * self.width
        if self.kind == "matmul_epilogue":
            M, N, K = self.rows, self.width, self.depth
            return 2 * (M * K + K * N + M * N) + 4 * N
        raise ValueError(self.kind)

    def label(self) -> str:
        if self.kind == "matmul_epilogue":
            return f"M={self.rows} K={self.depth} N={self.width} bias+gelu_tanh"
        if self.kind in ("transpose_th", "transpose_hd"):
            return f"T={self.rows} H={self.heads} D={D_HEAD}"
        if self.kind == "rope_2d":
            return f"T={self.rows} H={self.heads} D={D_HEAD}"
        return f"R={self.rows} C={self.width}"


# The per-kernel gate shapes of the benchmark's configuration 2 (seeded fp16
# N(0,1) inputs): the two block GEMMs with their fused bias + GELU epilogue
# at 256 tokens, the attention softmax over 12 x 256 x 256 scores, and the
# memory-bound kernels over 256 x 768 (rope and the transposes over
# [T, H, D] = [256, 12, 64]). At these sizes every kernel is launch-latency
# bound; the gates check the kernels there, the sweep measures bandwidth.
GATES = (
    Case("matmul_epilogue", 256, 768, depth=768),
    Case("matmul_epilogue", 256, 3072, depth=768),
    Case("softmax", 12 * 256, 256),
    Case("layernorm", 256, 768),
    Case("rmsnorm", 256, 768),
    Case("rope_2d", 256, 768, 12),
    Case("transpose_th", 256, 768, 12),
    Case("transpose_hd", 256, 768, 12),
    Case("add", 256, 768),
    Case("scale", 256, 768),
    Case("cast", 256, 768),
)


def cases(max_tensor_bytes: int = 4 << 30, kinds=KINDS) -> list[Case]:
    out = []
    for k in kinds:
        if k in ("transpose_th", "transpose_hd"):
            for t in TRANSPOSE_T:
                for h in TRANSPOSE_H:
                    out.append(Case(k, t, h * D_HEAD, h))
            continue
        for r in ROWS:
            for c in WIDTHS:
                if k == "rope_2d":
                    cs = Case(k, r, c, c // D_HEAD)
                else:
                    cs = Case(k, r, c)
                in_bytes = cs.elems * (4 if k == "cast" else 2)
                if in_bytes > max_tensor_bytes or cs.elems >= 1 << 31:
                    continue
                out.append(cs)
    return out


def _launcher(case: Case):
    """Allocate the case's tensors on the current device and return a
    zero-argument callable that launches the kernel once on the current
    stream (raising on a non-OK status)."""
    import torch
    L = _lib.lib()
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(1)
    R, C, k = case.rows, case.width, case.kind

    def f16(*shape):
        return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).half()

    def run(fn, *args):
        s = torch.cuda.current_stream().cuda_stream
        rc = fn(*args, s)
        if rc != 1:
            raise RuntimeError(f"{k} {case.label()}: status {_lib.status_name(rc)}")

    if k == "softmax":
        x, y = f16(R, C), torch.empty(R, C, device=dev, dtype=torch.half)
        return lambda: run(L.hexlib_b200_softmax_fp16, x.data_ptr(), y.data_ptr(), R, C), (x, y)
    if k == "layernorm":
        x, y = f16(R, C), torch.empty(R, C, device=dev, dtype=torch.half)
        w = 1 + 0.02 * torch.randn(C, generator=g, device=dev)
        b = 0.02 * torch.randn(C, generator=g, device=dev)
        return (lambda: run(L.hexlib_b200_layernorm_fp16, x.data_ptr(), w.data_ptr(),
                            b.data_ptr(), y.data_ptr(), R, C, ctypes.c_float(1e-6)),
                (x, y, w, b))
    if k == "rmsnorm":
        x, y, w = f16(R, C), torch.empty(R, C, device=dev, dtype=torch.half), f16(C)
        return (lambda: run(L.hexlib_b200_rmsnorm_fp16, x.data_ptr(), w.data_ptr(),
                            y.data_ptr(), R, C, ctypes.c_float(1e-6)), (x, y, w))
    if k == "rope_2d":
        H = case.heads
        x, y = f16(R, H, D_HEAD), torch.empty(R, H, D_HEAD, device=dev, dtype=torch.half)
        ang = torch.rand(R, D_HEAD, generator=g, device=dev) * 6.283
        ct, st = torch.cos(ang), torch.sin(ang)
        return (lambda: run(L.hexlib_b200_rope_2d_fp16, x.data_ptr(), ct.data_ptr(),
                            st.data_ptr(), y.data_ptr(), R, H, D_HEAD), (x, y, ct, st))
    if k == "add":
        a, b, y = f16(R, C), f16(R, C), torch.empty(R, C, device=dev, dtype=torch.half)
        return (lambda: run(L.hexlib_b200_add_fp16, a.data_ptr(), b.data_ptr(), y.data_ptr(),
                            R * C), (a, b, y))
    if k == "scale":
        x, y = f16(R, C), torch.empty(R, C, device=dev, dtype=torch.half)
        return (lambda: run(L.hexlib_b200_scale_fp16, x.data_ptr(), y.data_ptr(), R * C,
                            ctypes.c_float(0.125)), (x, y))
    if k == "cast":
        x = torch.randn(R, C, generator=g, device=dev)
        y = torch.empty(R, C, device=dev, dtype=torch.half)
        return lambda: run(L.hexlib_b200_cast_f32_f16, x.data_ptr(), y.data_ptr(), R * C), (x, y)
    if k == "transpose_th":
        H = case.heads
        x, y = f16(R, H, D_HEAD), torch.empty(H, R, D_HEAD, device=dev, dtype=torch.half)
        return (lambda: run(L.hexlib_b200_transpose_th_fp16, x.data_ptr(), y.data_ptr(), R, H,
                            D_HEAD), (x, y))
    if k == "transpose_hd":
        H = case.heads
        x, y = f16(H, R, D_HEAD), torch.empty(H, D_HEAD, R, device=dev, dtype=torch.half)
        return (lambda: run(L.hexlib_b200_transpose_hd_fp16, x.data_ptr(), y.data_ptr(), H, R,
                            D_HEAD), (x, y))
    if k == "matmul_epilogue":
        M, N, K = R, C, case.depth
        a = f16(M, K)
        w = (0.02 * torch.randn(K, N, generator=g, device=dev)).half()
        b = 0.02 * torch.randn(N, generator=g, device=dev)
        y = torch.empty(M, N, device=dev, dtype=torch.half)
        return (lambda: run(L.hexlib_b200_matmul_epilogue_fp16, a.data_ptr(), w.data_ptr(),
                            b.data_ptr(), y.data_ptr(), M, K, N, 1), (a, w, b, y))
    raise ValueError(k)


def time_case(case: Case, reps: int = 10, warmup: int = 3) -> float:
    """Median seconds of one launch."""
    import torch
    launch, keep = _launcher(case)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        launch()
    times = []
    for _ in range(reps):
        flush.fill_(1)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        # keep the stream busy while the host enqueues e0, the launch and e1,
        # so the timed pair holds the kernel and not the host's launch latency
        torch.cuda._sleep(200_000)
        e0.record()
        launch()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) / 1e3)
    del keep
    times.sort()
    return times[len(times) // 2]


def run(peak_gbs: float, max_tensor_bytes: int = 4 << 30, kinds=KINDS, reps: int = 10):
    """Yield one result dict per case."""
    for cs in cases(max_tensor_bytes, kinds):
        t = time_case(cs, reps=reps)
        gbs = cs.bytes / t / 1e9
        yield {"sweep": cs.kind, "shape": cs.label(), "bytes": cs.bytes,
               "us": round(t * 1e6, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak_gbs, 3)}
