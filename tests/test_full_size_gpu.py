"""GPU parity at the benchmark's full batch sizes, through properties that do
not need the CPU oracle to run at that scale:
  * after D2H, the whole host pool equals the pool that the reference's own
    transfer.cu (oracle/_ref, built from its source) produces for the same
    ids; both start from zeros;
  * D2H then H2D into zeroed GPU blocks restores the GPU blocks exactly.
Batches are the configurations' own (2048 blocks of Llama-3-8B with 50 %
joint runs; 1024 blocks of DeepSeek-V3 MLA with 128-block runs and
singletons); pools are smaller than the configurations' (ids are drawn
within them), which changes no kernel work per batch."""
import pytest
import torch

from kvcase import make_ids

pytestmark = pytest.mark.gpu

CASES = {
    # name: layers, heads, head_dim, tpb, mla, layout, gpu_blocks, cpu_blocks, batch, run_frac, max_run
    "cfg2_llama8b_layerwise": (32, 8, 128, 16, False, "LAYERWISE", 4096, 8192, 2048, 0.5, 64),
    "cfg2_llama8b_blockwise": (32, 8, 128, 16, False, "BLOCKWISE", 4096, 8192, 2048, 0.5, 64),
    "cfg5_dsv3_mla_blockwise": (61, 1, 576, 64, True, "BLOCKWISE", 2048, 4096, 1024, 0.5, 128),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_full_batch_matches_reference_kernel_and_round_trips(name):
    from flexkv_b200 import c_ext
    from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType, cpu_byte_strides, gpu_byte_strides
    from oracle import oracle as O
    if not O.reference_available():
        pytest.skip("oracle/_ref not built")
    L, H, D, tpb, mla, layout, ng, nc, n, frac, run = CASES[name]
    gl = KVCacheLayout(KVCacheLayoutType.LAYERWISE, L, ng, tpb, H, D, mla)
    cl = KVCacheLayout(KVCacheLayoutType[layout], L, nc, tpb, H, D, mla)
    gs, cs = gpu_byte_strides(gl, 2), cpu_byte_strides(cl, 2)
    gen = torch.Generator(device="cuda").manual_seed(11)
    per_layer = gl.kv_shape[1:]
    layers = [torch.randint(-2**15, 2**15, per_layer, dtype=torch.int16, device="cuda", generator=gen)
              for _ in range(L)]
    original = [x.clone() for x in layers]
    ptrs = torch.tensor([x.data_ptr() for x in layers], dtype=torch.int64)
    gids, cids = make_ids(n, ng, nc, 2024, frac, max_run=run)
    g_t, c_t = torch.from_numpy(gids), torch.from_numpy(cids)
    ours = torch.zeros(cl.get_total_elements(), dtype=torch.int16).pin_memory()
    ref = torch.zeros_like(ours).pin_memory()
    args = (gs["kv"], gs["block"])
    cargs = (cs["kv"], cs["layer"], cs["block"], gs["chunk"])
    c_ext.transfer_kv_blocks(g_t, ptrs, *args, c_t, ours, *cargs, 0, -1, False, False, mla)
    # the reference kernel reads ids and layer pointers from pinned host
    # memory while it runs: keep them referenced across the call
    g_pin, c_pin, p_pin = g_t.pin_memory(), c_t.pin_memory(), ptrs.pin_memory()
    rc = O.ref_lib().ref_transfer_kv_blocks(
        n, 0, L, g_pin.data_ptr(), p_pin.data_ptr(), args[0], args[1], c_pin.data_ptr(), ref.data_ptr(),
        cargs[0], cargs[1], cargs[2], 0, cargs[3], torch.cuda.current_stream().cuda_stream, 8, 0, 0, int(mla))
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(ours, ref), "host pool differs from the reference kernel's"
    assert bool((ours != 0).any())
    for x in layers:
        x[:, g_t.cuda()] = 0
    c_ext.transfer_kv_blocks(g_t, ptrs, *args, c_t, ours, *cargs, 0, -1, True, False, mla)
    torch.cuda.synchronize()
    for x, y in zip(layers, original):
        assert torch.equal(x, y)
