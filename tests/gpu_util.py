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


def argmax_margins(logits):
    """Per row: the oracle's top logit minus its runner-up (how far the row is
    from a tie that two accumulation orders could break differently)."""
    lg = np.asarray(logits, np.float32)
    part = np.partition(lg, -2, axis=-1)
    return part[..., -1] - part[..., -2]


def check_argmax_identical(got, logits, label=""):
    """The parity bar for the argmax: identical to the oracle's first-index
    argmax on every row.  The top-1 minus top-2 margins are printed, and a row
    whose margin is below one bf16 ulp of its top logit is named as a tie in
    the failure message (it still fails)."""
    ref = O.argmax_first(logits)
    marg = argmax_margins(logits)
    got = np.asarray(got).astype(np.int64).ravel()
    ref = np.asarray(ref).astype(np.int64).ravel()
    top = np.abs(np.max(np.asarray(logits, np.float32), axis=-1)).ravel()
    ties = [i for i in range(len(ref)) if marg.ravel()[i] < top[i] * 2.0 ** -7]
    print(f"{label} argmax margins: min {marg.min():.4g} median {np.median(marg):.4g}; "
          f"rows within one bf16 ulp: {ties}")
    bad = [i for i in range(len(ref)) if got[i] != ref[i]]
    assert not bad, (f"{label}: argmax differs on rows {bad} (got {[int(got[i]) for i in bad]}, oracle "
                     f"{[int(ref[i]) for i in bad]}, margins {[float(marg.ravel()[i]) for i in bad]}, ties {ties})")
