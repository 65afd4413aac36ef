"""GPU parity: kvm_restore_k (fused raw-K restore transform of stage-in:
dequant -> NeoX RoPE -> Walsh-Hadamard -> requant, src in device or mapped
pinned host memory) against the C restatement of the reference's kernels
(src/adapter/llama-kvmem-stagein.cu:104-234) and against the reference's own
stage-in route compiled from its source. Without RoPE every f32 step is rounded
identically: byte-exact. With RoPE, sincosf and the host's sinf / cosf (or the
reference's contracted multiply-adds) may differ in the last bits, which can move
a requantised code by one step."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import util as U

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kt", [U.Q8_0, U.Q4_0])
@pytest.mark.parametrize("n_rot,nrot", [(0, 0), (0, 128), (0, 512), (128, 256), (64, 64), (128, 0)])
def test_restore_k_matches_oracle(ctx, kt, n_rot, nrot):
    rng = np.random.default_rng(40 + kt + n_rot + nrot)
    n_head, dim = 4, 128
    theta = (10000.0 ** (-np.arange(0, dim, 2) / dim)).astype(np.float32)
    items = [(64, 0), (37, 4096), (128, 123457)]  # (tokens, pos0)
    dev = torch.device("cuda", 0)
    srcs, dsts, calls = [], [], []
    for i, (tokens, pos0) in enumerate(items):
        kb = U.make_k(rng, kt, 1, tokens, n_head, dim).reshape(-1)
        if i == 1:  # read straight from pinned host memory
            src_t = torch.from_numpy(kb.copy()).pin_memory()
        else:
            src_t = torch.from_numpy(kb.copy()).to(dev)
        dst_t = torch.zeros(kb.size, dtype=torch.uint8, device=dev)
        srcs.append((kb, src_t))
        dsts.append(dst_t)
        calls.append((src_t.data_ptr(), dst_t.data_ptr(), tokens, pos0))
    ctx.restore_k(kt, calls, n_head=n_head, head_dim=dim, n_rot=n_rot, theta=theta.tolist(), nrot=nrot)
    torch.cuda.synchronize()
    ctx.check_status("restore_k")
    for (tokens, pos0), (kb, _), dst_t in zip(items, srcs, dsts):
        rc, exp = O.restore_k(kt, kb, tokens=tokens, n_head=n_head, dim=dim, n_rot=n_rot, pos0=pos0, theta=theta,
                              nrot=nrot)
        assert rc == 0
        got = dst_t.cpu().numpy()
        if n_rot == 0:
            assert np.array_equal(got, exp), "restore transform differs from the oracle"
        else:
            a = U.decode_rows_f32(got.reshape(tokens * n_head, -1), kt, dim)
            b = U.decode_rows_f32(exp.reshape(tokens * n_head, -1), kt, dim)
            step = np.abs(b).max() / (7 if kt == U.Q4_0 else 100)
            assert np.abs(a - b).max() <= step
            assert np.mean(got == exp) > 0.97


@pytest.mark.parametrize("kt", [U.Q8_0, U.Q4_0])
@pytest.mark.parametrize("n_rot,nrot", [(0, 0), (0, 128), (0, 512), (128, 256), (64, 64), (128, 0)])
def test_restore_k_matches_reference_stagein(ctx, kt, n_rot, nrot):
    """kvm_restore_k against the reference's own stage-in route on the GPU: its
    kvmem_stagein_enqueue_k + kvmem_stagein_flush (slab H2D, dequant, NeoX RoPE with sincosf,
    Walsh-Hadamard, requant; src/adapter/llama-kvmem-stagein.cu:104-234, 673-881), compiled from
    its source into oracle/_ref/libkvref_cuda.so, on the same items; plus its V route (slab H2D
    and device copies) for byte records. Without RoPE byte-exact; with RoPE the reference's
    rotation is compiled with contracted multiply-adds, so a requantised code may move by one
    step where the f32 values differ in the last bit."""
    from oracle import oracle as Ox
    if Ox.ref_cuda() is None:
        pytest.fail("oracle/_ref/libkvref_cuda.so is missing (make -C oracle refcuda)")
    rng = np.random.default_rng(70 + kt + n_rot + nrot)
    n_head, dim = 4, 128
    theta = (10000.0 ** (-np.arange(0, dim, 2) / dim)).astype(np.float32)
    items = [(64, 0), (37, 4096), (128, 123457)]
    dev = torch.device("cuda", 0)
    ours, refs, k_items, calls, hosts = [], [], [], [], []
    for tokens, pos0 in items:
        kb = U.make_k(rng, kt, 1, tokens, n_head, dim).reshape(-1)
        src = torch.from_numpy(kb.copy()).to(dev)
        o = torch.zeros(kb.size, dtype=torch.uint8, device=dev)
        r = torch.zeros(kb.size, dtype=torch.uint8, device=dev)
        hosts.append(src)
        ours.append(o)
        refs.append(r)
        calls.append((src.data_ptr(), o.data_ptr(), tokens, pos0))
        k_items.append((kb, r.data_ptr(), tokens, pos0))
    v = rng.integers(0, 256, 4608, dtype=np.uint8)
    v_dst = torch.zeros(v.size, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    Ox.ref_stagein(kt, k_items, n_head=n_head, dim=dim, n_rot=n_rot, theta=theta if n_rot else None, nrot=nrot,
                   v_items=[(v, v_dst.data_ptr())])
    ctx.restore_k(kt, calls, n_head=n_head, head_dim=dim, n_rot=n_rot, theta=theta.tolist(), nrot=nrot)
    torch.cuda.synchronize()
    ctx.check_status("restore_k")
    assert np.array_equal(v_dst.cpu().numpy(), v)
    for (tokens, _), o, r in zip(items, ours, refs):
        got, want = o.cpu().numpy(), r.cpu().numpy()
        if n_rot == 0:
            assert np.array_equal(got, want), "restore transform differs from the reference's stage-in"
        else:
            a = U.decode_rows_f32(got.reshape(tokens * n_head, -1), kt, dim)
            b = U.decode_rows_f32(want.reshape(tokens * n_head, -1), kt, dim)
            step = np.abs(b).max() / (7 if kt == U.Q4_0 else 100)
            assert np.abs(a - b).max() <= step
            assert np.mean(got == want) > 0.97


def test_restore_k_rejects_bad_shapes(ctx):
    import kvmem_b200 as K
    dev = torch.device("cuda", 0)
    buf = torch.zeros(4 * 34 * 4, dtype=torch.uint8, device=dev)
    item = [(buf.data_ptr(), buf.data_ptr(), 1, 0)]
    with pytest.raises(K.KvmError) as e:
        ctx.restore_k(U.F16, item, n_head=4, head_dim=32)
    assert e.value.code == K._abi.ERR_UNSUPPORTED
    with pytest.raises(K.KvmError) as e:  # nrot must be 64..512 and divide the row
        ctx.restore_k(U.Q8_0, item, n_head=4, head_dim=32, nrot=96)
    assert e.value.code == K._abi.ERR_INVALID_ARGUMENT
    with pytest.raises(K.KvmError) as e:  # n_rot beyond the head
        ctx.restore_k(U.Q8_0, item, n_head=4, head_dim=32, n_rot=64, theta=[1.0] * 32)
    assert e.value.code == K._abi.ERR_INVALID_ARGUMENT
