"""Runs the per-column scans (float32 forward and backward, the backward into
the fp16 split, and the bf16-storage pair) on a seeded problem and saves every
output to the file named by argv[1].  tests/test_gpu_scan_units.py runs it
twice, as child processes with HS_SCAN_UNITS=1 and =2 (the variable is read
once per process), and compares the two files bit for bit."""

import sys

import torch


def main(path, T, B, H):
    from prlstm_b200 import _lib as L

    dev = torch.device("cuda", 0)
    lib = L.load()
    P, st, sw = L.ptr, L.stream_ptr(dev), L.status_word(dev)
    g = torch.Generator(device=dev).manual_seed(T * 7 + B * 3 + H)
    z = torch.randn(T, B, 4 * H, device=dev, generator=g) * 3
    z[..., H:2 * H] += 4.0
    c0 = torch.rand(B, H, device=dev, generator=g)
    dout = torch.randn(T, B, H, device=dev, generator=g)
    dh_n = torch.randn(B, H, device=dev, generator=g)
    dc_n = torch.randn(B, H, device=dev, generator=g)
    res = {}
    ws = L.workspace(max(lib.hs_scan_workspace_bytes(T, B, H), lib.hs_scan_split_workspace_bytes(T, B, H)), dev)
    out, c = torch.empty(T, B, H, device=dev), torch.empty(T, B, H, device=dev)
    hn, cn = torch.empty(B, H, device=dev), torch.empty(B, H, device=dev)
    kf = torch.zeros(1, dtype=torch.int32, device=dev)
    L.call("hs_scan_forward_kf", P(z), P(c0), P(out), P(c), P(hn), P(cn), T, B, H, 1e-6, P(ws), ws.numel(), P(kf),
           P(sw), st)
    res.update(out=out, c=c, h_n=hn, c_n=cn, kf=kf.clone())
    dz, dc0, db = torch.empty_like(z), torch.empty(B, H, device=dev), torch.empty(4 * H, device=dev)
    L.call("hs_scan_backward", P(z), P(c), P(c0), P(dout), P(dh_n), P(dc_n), P(dz), P(dc0), P(db), T, B, H, 1e-6,
           P(ws), ws.numel(), P(sw), st)
    res.update(dz=dz, dc0=dc0, db=db)
    split = torch.empty(lib.hs_split_bytes(T * B, 4 * H), dtype=torch.uint8, device=dev)
    scale = torch.zeros(64, dtype=torch.int32, device=dev)
    dc0s, dbs = torch.empty(B, H, device=dev), torch.empty(4 * H, device=dev)
    zc = z.clone()
    L.call("hs_scan_backward_split", P(zc), P(c), P(c0), P(dout), P(dh_n), P(dc_n), P(kf), P(split), P(scale),
           P(dc0s), P(dbs), T, B, H, 1e-6, P(ws), ws.numel(), P(sw), st)
    res.update(split=split, scale=scale[:1].clone(), dc0_split=dc0s, db_split=dbs)
    if H % 8 == 0 and lib.hs_scan_uses_column_kernels(T, B, H):
        bf = torch.bfloat16
        zb, db16 = z.to(bf), dout.to(bf)
        ob, cb = torch.empty(T, B, H, device=dev, dtype=bf), torch.empty(T, B, H, device=dev, dtype=bf)
        hb, cnb = torch.empty(B, H, device=dev), torch.empty(B, H, device=dev)
        L.call("hs_scan_forward_bf16", P(zb), P(c0), P(ob), P(cb), P(hb), P(cnb), T, B, H, 1e-6, P(sw), st)
        dzb = torch.empty(T, B, 4 * H, device=dev, dtype=bf)
        dc0b, dbb = torch.empty(B, H, device=dev), torch.empty(4 * H, device=dev)
        wsb = L.workspace(lib.hs_scan_bf16_workspace_bytes(T, B, H), dev)
        L.call("hs_scan_backward_bf16", P(zb), P(cb), P(c0), P(db16), P(dh_n), P(dc_n), P(dzb), P(dc0b), P(dbb), T, B,
               H, 1e-6, P(wsb), wsb.numel(), P(sw), st)
        res.update(bf_out=ob, bf_c=cb, bf_h_n=hb, bf_c_n=cnb, bf_dz=dzb, bf_dc0=dc0b, bf_db=dbb)
    torch.cuda.synchronize(dev)
    L.check_device_status(dev)
    torch.save({k: v.cpu() for k, v in res.items()}, path)


if __name__ == "__main__":
    main(sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4]))
