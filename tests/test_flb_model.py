"""FLBTransformer (flb_model/) against the reference FLB_Transformer's outputs and gradients
(tests/golden/flb_model.pt, made by running the reference on CPU), and its greedy decode."""
import pytest
import torch
import torch.nn.functional as F


def _model(c, device="cpu"):
    from flb_model import FLBTransformer
    return FLBTransformer(c["vocab"], hidden_dim=c["hidden"], num_layers=c["layers"],
                          seq_len=c["seq_len"], batch_size=c["batch"]).to(device)


def test_state_dict_layout_matches_reference(flb_golden):
    """Same parameter and buffer names and shapes as the reference model: checkpoints load
    either way (strict)."""
    m = _model(flb_golden["config"])
    ref = flb_golden["state_dict"]
    mine = m.state_dict()
    assert set(mine) == set(ref)
    for k, v in ref.items():
        assert mine[k].shape == v.shape, k
    m.load_state_dict(ref, strict=True)


@pytest.mark.gpu
def test_flb_model_matches_reference(cuda, flb_golden):
    """fp32 end to end with tanh.approx attention: logits, aux loss, next contexts and every
    parameter gradient of cross-entropy + aux within 2e-3 of the reference (relative to each
    tensor's magnitude for gradients)."""
    g = flb_golden
    c = g["config"]
    m = _model(c, cuda)
    m.load_state_dict(g["state_dict"])
    m.eval()
    logits, aux, (lat, fdbk) = m(g["tokens"].to(cuda))
    assert torch.allclose(logits.cpu(), g["logits"], atol=2e-3)
    assert abs(aux.item() - g["aux_loss"].item()) < 2e-3 * max(1.0, g["aux_loss"].abs().item())
    assert torch.allclose(lat.cpu(), g["next_lat"], atol=2e-3)
    assert torch.allclose(fdbk.cpu(), g["next_fdbk"], atol=2e-3)
    loss = F.cross_entropy(logits.reshape(-1, c["vocab"]), g["targets"].to(cuda).reshape(-1)) + aux
    loss.backward()
    for k, p in m.named_parameters():
        if k not in g["grads"]:
            assert p.grad is None or not p.grad.any(), k
            continue
        ref = g["grads"][k]
        scale = max(ref.abs().max().item(), 1e-3)
        assert (p.grad.cpu() - ref).abs().max().item() <= 2e-3 * scale, k


@pytest.mark.gpu
def test_flb_model_graphed_engine_matches_eager(cuda, flb_golden):
    """The model through a GraphedWavefrontEngine (forward + backward captured) gives the eager
    engine's logits and gradients."""
    g = flb_golden
    c = g["config"]
    ma, mb = _model(c, cuda), _model(c, cuda)
    ma.load_state_dict(g["state_dict"])
    mb.load_state_dict(g["state_dict"])
    ma.eval()
    mb.eval()
    tok = g["tokens"].to(cuda)
    graphed = mb.engine.graphed(mb.embedding(tok).detach())
    for _ in range(2):
        la, aa, _ = ma(tok)
        lb, ab, _ = mb(tok, engine=graphed)
        assert torch.allclose(la, lb, atol=1e-5)
        (la.square().mean() + aa).backward()
        (lb.square().mean() + ab).backward()
    for (ka, pa), (kb, pb) in zip(ma.named_parameters(), mb.named_parameters()):
        if pa.grad is None:
            assert pb.grad is None or not pb.grad.any(), ka
            continue
        scale = max(pa.grad.abs().max().item(), 1e-3)
        assert (pa.grad - pb.grad).abs().max().item() <= 1e-4 * scale, ka


@pytest.mark.gpu
def test_greedy_decode_graphed_equals_eager(cuda):
    from flb_model import FLBTransformer, greedy_decode
    torch.manual_seed(5)
    m = FLBTransformer(50, hidden_dim=64, num_layers=3, seq_len=8, batch_size=2).to(cuda).eval()
    with torch.no_grad():
        for layer in m.layers:
            layer.flb_attention.v_a.normal_(0.0, 0.5)
    prompt = torch.randint(0, 50, (2, 8), device=cuda)
    a = greedy_decode(m, prompt, 5, graphed=False)
    b = greedy_decode(m, prompt, 5, graphed=True)
    assert a.shape == (2, 5)
    assert torch.equal(a, b)
    # the first generated token is the argmax of the prompt's last-position logits
    with torch.no_grad():
        logits, _, _ = m(prompt)
    assert torch.equal(a[:, 0], logits[:, -1].argmax(-1))


def _bf16_model(seed, V=50, D=64, L=4, S=6, B=3, heads=8):
    from flb_model import FLBTransformer
    torch.manual_seed(seed)
    m = FLBTransformer(V, hidden_dim=D, num_layers=L, seq_len=S, batch_size=B,
                       num_heads=heads).cuda().eval()
    with torch.no_grad():
        for name, p in m.named_parameters():
            if name.endswith("v_a"):
                p.normal_(0.0, 0.5)
            elif "bias" in name and "norm" not in name:
                p.normal_(0.0, 0.1)
    return m


def _max_rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6)).item()


@pytest.mark.gpu
@pytest.mark.parametrize("D,B", [(64, 3), (96, 20), (80, 4)])
def test_native_flb_forward_matches_generic_path(cuda, D, B):
    """Inference under bf16 autocast: the native whole-grid forward (flb_block_grid_fwd) against
    the per-tick vmapped path of the same engine: every port grid, logits and contexts, at
    several d_model and batch sizes (batch 20: more rows per cell than the end-to-end shape's 16;
    d_model 80 and 96: not powers of two)."""
    m = _bf16_model(7, D=D, B=B)
    tok = torch.randint(0, 50, (B, 6), device=cuda)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        x = m.embedding(tok)
        m.engine.native_cells = False
        gen = [g.clone() for g in m.engine(x)]
        lg, ag, cg = m(tok)
        m.engine.native_cells = True
        nat_ = [g.clone() for g in m.engine(x)]
        ln_, an, cn = m(tok)
    for p in range(4):
        assert nat_[p].dtype == torch.bfloat16
        assert _max_rel(nat_[p], gen[p]) < 3e-2, p
    assert _max_rel(ln_, lg) < 3e-2
    assert abs(an.item() - ag.item()) <= 3e-2 * abs(ag.item()) + 1e-6
    for a, b in zip(cn, cg):
        assert _max_rel(a, b) < 3e-2


@pytest.mark.gpu
def test_native_flb_forward_e2e_cell_shape(cuda):
    """Batch 16, d_model 768, 12 heads (the end-to-end configuration's cell) through the native
    whole-grid forward: every port grid, the logits and the contexts against the per-tick
    vmapped path of the same engine under bf16 autocast (3e-2 relative to each tensor's largest
    magnitude), and the CUDA-graph replay of the native forward against eager (equal)."""
    from wavefront.wavefront_graph import GraphedWavefrontEngine
    m = _bf16_model(23, D=768, L=6, S=5, B=16, heads=12)
    tok = torch.randint(0, 50, (16, 5), device=cuda)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        x = m.embedding(tok)
        # the native path first, on the engine's freshly allocated (zero) grids, so that nothing
        # the per-tick path leaves in the shared buffers can stand in for its outputs
        nat_ = [g.clone() for g in m.engine(x)]
        ln_, an, cn = m(tok)
        m.engine.native_cells = False
        gen = [g.clone() for g in m.engine(x)]
        lg, ag, cg = m(tok)
        m.engine.native_cells = True
        graphed = GraphedWavefrontEngine(m.engine, x, backward=False)
        assert graphed.native_flb
        lgr, _, _ = m(tok, engine=graphed)
    for p in range(4):
        assert torch.isfinite(nat_[p].float()).all(), p
        assert _max_rel(nat_[p], gen[p]) < 3e-2, (p, _max_rel(nat_[p], gen[p]))
    assert _max_rel(ln_, lg) < 3e-2
    assert abs(an.item() - ag.item()) <= 3e-2 * abs(ag.item()) + 1e-6
    for a, b in zip(cn, cg):
        assert _max_rel(a, b) < 3e-2
    assert torch.equal(lgr, ln_)


@pytest.mark.gpu
def test_native_flb_forward_against_reference(cuda, flb_golden):
    """The native path (bf16) against the reference model in fp32 on the golden case: logits
    within 2e-2 of the reference relative to their largest magnitude (the bf16 tolerance; the
    per-tick path at the same precision is shown beside it)."""
    g = flb_golden
    c = g["config"]
    m = _model(c, cuda)
    m.load_state_dict(g["state_dict"])
    m.eval()
    tok = g["tokens"].to(cuda)
    ref = g["logits"].to(cuda)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        m.engine.native_cells = False
        lg, _, _ = m(tok)
        m.engine.native_cells = True
        ln_, _, _ = m(tok)
    e_gen, e_nat = _max_rel(lg, ref), _max_rel(ln_, ref)
    assert e_nat < 2e-2, (e_nat, e_gen)


@pytest.mark.gpu
def test_native_flb_decode_graphed_equals_eager(cuda):
    """Greedy decode under bf16 autocast: the CUDA-graph replay of the native forward gives the
    same tokens as eager native forwards."""
    from flb_model import greedy_decode
    m = _bf16_model(9, S=8, B=2)
    prompt = torch.randint(0, 50, (2, 8), device=cuda)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        a = greedy_decode(m, prompt, 6, graphed=False)
        b = greedy_decode(m, prompt, 6, graphed=True)
    assert torch.equal(a, b)


def _train_grads(m, tok, targets, native):
    m.engine.native_cells = native
    m.zero_grad(set_to_none=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits, aux, _ = m(tok)
    loss = F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), targets.reshape(-1)) + aux
    loss.backward()
    return {k: p.grad.detach().float().clone() for k, p in m.named_parameters()
            if p.grad is not None}, loss.item()


@pytest.mark.gpu
def test_native_flb_training_matches_generic_path(cuda):
    """Training under bf16 autocast: the native backward (flb_block_grid_bwd) against the
    per-tick vjp path of the same engine — loss and every parameter gradient, the embedding's
    included (it carries dx)."""
    m = _bf16_model(13)
    tok = torch.randint(0, 50, (3, 6), device=cuda)
    targets = torch.randint(0, 50, (3, 6), device=cuda)
    gn, ln_ = _train_grads(m, tok, targets, True)
    gg, lg = _train_grads(m, tok, targets, False)
    assert abs(ln_ - lg) <= 2e-2 * abs(lg)
    assert set(gn) == set(gg)
    for k in gg:
        assert _max_rel(gn[k], gg[k]) < 6e-2, (k, _max_rel(gn[k], gg[k]))


@pytest.mark.gpu
@pytest.mark.parametrize("D,L,S,B,H", [(64, 4, 6, 3, 8), (768, 4, 5, 16, 12)])
def test_native_flb_training_saved_matches_recompute(cuda, D, L, S, B, H):
    """The native backward restoring the forward's per-cell intermediates
    (flb_block_grid_fwd_save / flb_block_grid_bwd_saved, the default) against the same backward
    recomputing each tick's forward stages (engine.native_flb_save = False): loss and every
    parameter gradient within 2e-2 of the largest magnitude (the two forwards round z_l and the
    LayerNorm statistics differently in the last bit)."""
    m = _bf16_model(19, D=D, L=L, S=S, B=B, heads=H)  # eval mode: no dropout
    tok = torch.randint(0, 50, (B, S), device=cuda)
    targets = torch.randint(0, 50, (B, S), device=cuda)
    gs, ls = _train_grads(m, tok, targets, True)
    assert m.engine.graph_workspace["flb_saved"].numel() > 0
    m.engine.native_flb_save = False
    gr, lr = _train_grads(m, tok, targets, True)
    assert abs(ls - lr) <= 2e-2 * abs(lr)
    assert set(gs) == set(gr)
    for k in gr:
        assert _max_rel(gs[k], gr[k]) < 2e-2, (k, _max_rel(gs[k], gr[k]))


@pytest.mark.gpu
def test_native_flb_training_against_reference(cuda, flb_golden):
    """Native bf16 gradients against the reference model's fp32 gradients (golden): every
    parameter's gradient within 2e-2 of the reference relative to the tensor's largest
    magnitude, the bf16 tolerance (measured worst 0.016; the per-tick path's 0.017)."""
    g = flb_golden
    c = g["config"]
    m = _model(c, cuda)
    m.load_state_dict(g["state_dict"])
    m.eval()
    tok, targets = g["tokens"].to(cuda), g["targets"].to(cuda)
    gn, _ = _train_grads(m, tok, targets, True)
    gg, _ = _train_grads(m, tok, targets, False)
    for k, ref in g["grads"].items():
        ref = ref.to(cuda)
        e_nat, e_gen = _max_rel(gn[k], ref), _max_rel(gg[k], ref)
        assert e_nat < 2e-2, (k, e_nat, e_gen)


@pytest.mark.gpu
def test_native_flb_graphed_training_matches_eager(cuda):
    """The native FLB forward and backward captured by GraphedWavefrontEngine give the eager
    native path's loss and gradients, over two steps with an in-place parameter update."""
    ma = _bf16_model(17)
    mb = _bf16_model(17)
    tok = torch.randint(0, 50, (3, 6), device=cuda)
    targets = torch.randint(0, 50, (3, 6), device=cuda)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        graphed = mb.engine.graphed(mb.embedding(tok).detach())
    assert graphed.native_flb
    for step in range(2):
        outs = []
        for m, eng in ((ma, None), (mb, graphed)):
            m.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                logits, aux, _ = m(tok, engine=eng)
            loss = F.cross_entropy(logits.float().reshape(-1, 50), targets.reshape(-1)) + aux
            loss.backward()
            outs.append((loss.item(), {k: p.grad.float().clone() for k, p in m.named_parameters()
                                       if p.grad is not None}))
        (la, ga), (lb, gb) = outs
        assert abs(la - lb) <= 1e-3 * abs(la)
        assert set(ga) == set(gb)
        for k in ga:
            assert _max_rel(gb[k], ga[k]) < 1e-2, (step, k)
        with torch.no_grad():
            for pa, pb in zip(ma.parameters(), mb.parameters()):
                pa.mul_(0.95)
                pb.mul_(0.95)
