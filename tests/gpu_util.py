"""Helpers for the GPU parity tests: device buffers (torch is only plumbing
here) and the comparison metrics of the parity bar."""
import numpy as np

from oracle import iam_oracle as O


def dev(a, torch, dtype=None):
    """numpy array -> CUDA tensor with the same bits."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        t = torch.from_numpy(a.view(np.int16)).cuda()
    elif a.dtype == np.uint32:
        t = torch.from_numpy(a.view(np.int32)).cuda()
    else:
        t = torch.from_numpy(a).cuda()
    return t


def host_u16(t):
    return t.cpu().numpy().view(np.uint16)


def empty_u16(torch, *shape):
    return torch.empty(shape, dtype=torch.int16, device="cuda")


def ptr(t):
    return t.data_ptr()


def rel_err(got, ref):
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def cosine(got, ref):
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    return float(got @ ref / max(np.linalg.norm(got) * np.linalg.norm(ref), 1e-30))


def assert_close_bf16(got_u16, ref_f32, rel=1e-2, cos=0.9999):
    g = O.from_u16(got_u16)
    assert np.all(np.isfinite(g))
    r = rel_err(g, ref_f32)
    c = cosine(g, ref_f32)
    assert r <= rel and c >= cos, f"rel_err={r:.3g} cos={c:.6f}"
    return r, c
