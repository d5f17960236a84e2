"""Streaming VAE decode (waveforcing_b200/pipelines/vae.py) on CPU.

* Parity with the reference's own Wan2.1 VAE decoder
  (naive_rt/rolling_forcing/wan/modules/vae.py, ``WanVAE_.decode``), imported
  from a WaveForcing checkout, with this module's random weights copied into
  it: small widths, a 5-frame latent.
* Chunked pushes equal the frame-by-frame decode.
* 1 + 4 (F - 1) pixel frames.
* The contiguous FLOP-balanced unit partition.
* A 3-rank gloo pipeline (the reference's ``vae_stage``) equals one process.
"""

import importlib.util
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from baseline import harness
from waveforcing_b200.pipelines import vae as V

CFG = V.VAEConfig(dim=8, z_dim=4)


def _ref_vae_module():
    root = harness.reference_checkout()
    cands = [os.path.join(c, "naive_rt", "rolling_forcing", "wan", "modules", "vae.py")
             for c in ([root] if root else []) + [os.path.join(os.path.dirname(harness.ROOT), "reference")]]
    for path in cands:
        if os.path.isfile(path):
            spec = importlib.util.spec_from_file_location("ref_wan_vae", path)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            return mod
    return None


def _load_into_reference(ours: V.VAEDecoder, ref) -> None:
    """Copy our weights into the reference's WanVAE_ under its names."""
    names = {name: (t, shape) for t, name, shape in ours.reference_names().values()}
    missing = set(k for k, _ in ref.named_parameters() if k.startswith("decoder.") or k.startswith("conv2.")) - set(names)
    assert not missing, missing
    with torch.no_grad():
        for k, p in ref.named_parameters():
            if k in names:
                t, shape = names[k]
                v = t.reshape(shape) if shape else t
                assert tuple(p.shape) == tuple(v.shape), (k, p.shape, v.shape)
                p.copy_(v)


def test_decoder_matches_reference_wan_vae():
    mod = _ref_vae_module()
    if mod is None:
        pytest.skip("needs a WaveForcing checkout (naive_rt/rolling_forcing/wan/modules/vae.py)")
    ours = V.VAEDecoder.random(CFG, seed=3)
    ref = mod.WanVAE_(dim=CFG.dim, z_dim=CFG.z_dim, dim_mult=list(CFG.dim_mult), num_res_blocks=CFG.num_res_blocks,
                      attn_scales=[], temperal_downsample=list(reversed(CFG.temporal_upsample))).eval()
    _load_into_reference(ours, ref)
    g = torch.Generator().manual_seed(5)
    z = torch.randn(1, CFG.z_dim, 5, 4, 6, generator=g)
    scale = [ours.units[0].mean.detach().clone(), ours.units[0].inv_std.detach().clone()]
    with torch.no_grad():
        want = ref.decode(z, scale).clamp(-1, 1)[0]
    got = V.decode_framewise(ours, z)
    assert tuple(got.shape) == (3, 1 + 4 * 4, 32, 48) == tuple(want.shape)
    assert float(want.abs().max()) > 0.05
    assert torch.allclose(got, want, atol=2e-5, rtol=1e-4), float((got - want).abs().max())
    # the stream fed whole chunks (frame 0 alone, then the rest) gives the same pixels
    s = V.DecodeStream(ours)
    chunked = torch.cat([s.push(z[:, :, :3]), s.push(z[:, :, 3:])], 1)
    assert torch.allclose(chunked, want, atol=2e-5, rtol=1e-4)
    # the drop-in direction: a decoder built from the reference module's weights and latent statistics
    again = V.VAEDecoder.from_reference(ref, scale[0], 1.0 / scale[1], CFG)
    assert torch.allclose(V.decode_framewise(again, z), got, atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("pushes", [[1, 3, 1], [3, 3], [2, 1, 1, 2]])
def test_chunked_pushes_equal_framewise(pushes):
    dec = V.VAEDecoder.random(CFG, seed=1)
    F_ = sum(pushes)
    z = torch.randn(CFG.z_dim, F_, 3, 5, generator=torch.Generator().manual_seed(2))
    want = V.decode_framewise(dec, z)
    s = V.DecodeStream(dec)
    outs, f0 = [], 0
    for n in pushes:
        outs.append(s.push(z[:, f0:f0 + n]))
        f0 += n
    got = torch.cat(outs, 1)
    assert tuple(got.shape) == (3, 1 + 4 * (F_ - 1), 24, 40)
    assert torch.allclose(got, want, atol=1e-5, rtol=1e-5)


def test_partition_units_is_balanced_and_contiguous():
    import itertools

    costs = [1, 1, 1, 10, 1, 1, 5, 5]
    cuts = V.partition_units(costs, 3)
    assert cuts[0] == 0 and cuts[-1] == len(costs) and cuts == sorted(cuts)
    best = min(max(sum(costs[a:b]) for a, b in zip((0,) + c, c + (len(costs),)))
               for c in itertools.combinations(range(1, len(costs)), 2))
    assert max(sum(costs[a:b]) for a, b in zip(cuts, cuts[1:])) == best == 11
    dec = V.VAEDecoder(V.VAEConfig())
    f = dec.unit_flops(60, 104)
    assert len(f) == len(dec.units) and all(x > 0 for x in f)
    # the full-resolution stage dominates: the head and the last stage's blocks
    assert sum(f[-4:]) > 0.3 * sum(f)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dec = V.VAEDecoder.random(CFG, seed=4)
        cuts = V.partition_units(dec.unit_flops(3, 5), world)
        st = V.VAEPipelineStage(dec, cuts, rank, list(range(world)))
        z = torch.randn(CFG.z_dim, 7, 3, 5, generator=torch.Generator().manual_seed(9))
        if rank == 0:
            for a, b in ((0, 3), (3, 6), (6, 7)):  # three chunks as the store finishes them
                for y in st.push_latents(z[:, a:b]):
                    st.send_next(y)
            st.send_next(None)
            q.put((rank, cuts, None))
        else:
            outs = st.serve()
            # numpy, not a tensor: a queued tensor's shared storage dies with its sender
            q.put((rank, cuts, torch.cat(outs, 1).numpy() if outs else None))
    except Exception as e:  # report instead of hanging the others
        q.put((rank, repr(e), None))
    finally:
        dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_pipeline_over_three_ranks_equals_one_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r, cuts, out = q.get(timeout=180)
        assert not isinstance(cuts, str), cuts
        res[r] = (cuts, out)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    cuts = res[0][0]
    assert len(cuts) == 4 and all(b > a for a, b in zip(cuts, cuts[1:]))
    dec = V.VAEDecoder.random(CFG, seed=4)
    z = torch.randn(CFG.z_dim, 7, 3, 5, generator=torch.Generator().manual_seed(9))
    s = V.DecodeStream(dec)
    want = torch.cat([s.push(z[:, a:b]) for a, b in ((0, 3), (3, 6), (6, 7))], 1)
    got = torch.from_numpy(res[2][1]) if res[2][1] is not None else None
    assert got is not None and tuple(got.shape) == tuple(want.shape) == (3, 25, 24, 40)
    assert torch.equal(got, want)
