"""Value and gradient of every objective against an independent fp64 restatement.

Each oracle below is written element by element (Python loops over rows,
pairs or triplets, in float64) from the Sentence-Transformers definition the
reference reproduces (src/representax/tasks/*/losses.py); the library's
vectorised fp32 version must agree in value and in its gradient with respect
to the embeddings. Parity model: tests/tasks/test_sentence_transformers_parity.py
and the per-family tests of the reference.
"""

import math

import pytest
import torch

from representax_b200.tasks import objectives as O

TOL = dict(rtol=2e-5, atol=2e-6)


def _leaf(*shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g, dtype=torch.float64) * scale).requires_grad_(True)


def _check(fn_impl, fn_oracle, inputs, tol=TOL):
    """Compare value and input gradients of the fp32 implementation with the fp64 oracle."""

    impl_in = [x.detach().float().requires_grad_(x.requires_grad) for x in inputs]
    got = fn_impl(*impl_in)
    want = fn_oracle(*inputs)
    assert math.isclose(float(got), float(want), rel_tol=tol["rtol"] * 10, abs_tol=tol["atol"] * 10), (
        float(got), float(want))
    diff_in = [(a, b) for a, b in zip(impl_in, inputs) if b.requires_grad]
    grads_got = torch.autograd.grad(got, [a for a, _ in diff_in], allow_unused=True)
    grads_want = torch.autograd.grad(want, [b for _, b in diff_in], allow_unused=True)
    for g1, g2 in zip(grads_got, grads_want):
        if g2 is None:
            assert g1 is None or torch.count_nonzero(g1) == 0
            continue
        torch.testing.assert_close(g1.double(), g2, rtol=tol["rtol"] * 50, atol=tol["atol"] * 50)


def _cos(a, b):
    return (a * b).sum() / (a.norm() * b.norm())


def _dist(a, b, metric):
    if metric == "cosine":
        return 1 - _cos(a, b)
    diff = a - b + 1e-6
    return diff.norm() if metric == "euclidean" else diff.abs().sum()


# ------------------------------------------------------------------ pairwise (K3)
def test_cosine_regression():
    u, v = _leaf(7, 5, seed=1), _leaf(7, 5, seed=2)
    y = torch.rand(7, generator=torch.Generator().manual_seed(3), dtype=torch.float64)

    def oracle(u, v):
        return sum((_cos(u[i], v[i]) - y[i]) ** 2 for i in range(7)) / 7

    _check(lambda a, b: O.cosine_regression_loss(a, b, y.float()), oracle, [u, v])


@pytest.mark.parametrize("metric", ["cosine", "euclidean", "manhattan"])
def test_contrastive(metric):
    u, v = _leaf(8, 4, seed=4, scale=0.3), _leaf(8, 4, seed=5, scale=0.3)
    y = torch.tensor([1, 0, 1, 0, 0, 1, 1, 0], dtype=torch.float64)
    margin = 0.5 if metric == "cosine" else 1.5

    def oracle(u, v):
        total = 0
        for i in range(8):
            d = _dist(u[i], v[i], metric)
            total = total + 0.5 * (y[i] * d ** 2 + (1 - y[i]) * torch.clamp(margin - d, min=0) ** 2)
        return total / 8

    _check(lambda a, b: O.contrastive_loss(a, b, y.float(), metric=metric, margin=margin), oracle, [u, v])


@pytest.mark.parametrize("metric", ["cosine", "euclidean"])
def test_online_contrastive(metric):
    u, v = _leaf(10, 4, seed=6, scale=0.5), _leaf(10, 4, seed=7, scale=0.5)
    y = torch.tensor([1, 0, 1, 0, 0, 1, 1, 0, 1, 0], dtype=torch.float64)
    margin = 0.5 if metric == "cosine" else 2.0

    def oracle(u, v):
        d = [_dist(u[i], v[i], metric) for i in range(10)]
        pos = [d[i] for i in range(10) if y[i] == 1]
        neg = [d[i] for i in range(10) if y[i] == 0]
        neg_cut = max(float(x) for x in pos) if len(pos) > 1 else sum(float(x) for x in neg) / len(neg)
        pos_cut = min(float(x) for x in neg) if len(neg) > 1 else sum(float(x) for x in pos) / len(pos)
        total = 0
        for x in pos:
            if float(x) > pos_cut:
                total = total + x ** 2
        for x in neg:
            if float(x) < neg_cut:
                total = total + torch.clamp(margin - x, min=0) ** 2
        return total

    _check(lambda a, b: O.online_contrastive_loss(a, b, y.float(), metric=metric, margin=margin), oracle, [u, v])


def _angle(a, b):
    half = a.shape[0] // 2
    re_a, im_a, re_b, im_b = a[:half], a[half:], b[:half], b[half:]
    denom = (re_b ** 2 + im_b ** 2).sum()
    real = (re_a * re_b + im_a * im_b) / denom
    imag = (im_a * re_b - re_a * im_b) / denom
    ratio = (re_a ** 2 + im_a ** 2).sum().sqrt() / (re_b ** 2 + im_b ** 2).sum().sqrt()
    return ((real / ratio).sum() + (imag / ratio).sum()).abs()


@pytest.mark.parametrize("similarity", ["cosine", "angle"])
def test_cosent_and_angle(similarity):
    u, v = _leaf(6, 8, seed=8), _leaf(6, 8, seed=9)
    y = torch.tensor([0.1, 0.9, 0.5, 0.3, 0.7, 0.2], dtype=torch.float64)
    scale = 20.0

    def oracle(u, v):
        sim = _cos if similarity == "cosine" else _angle
        s = [sim(u[i], v[i]) * scale for i in range(6)]
        terms = [torch.zeros((), dtype=torch.float64)]
        terms += [s[i] - s[j] for i in range(6) for j in range(6) if y[i] < y[j]]
        return torch.logsumexp(torch.stack(terms), 0)

    _check(lambda a, b: O.pair_ranking_loss(a, b, y.float(), scale=scale, similarity=similarity), oracle, [u, v])


# ------------------------------------------------------------------ triplet (K4)
@pytest.mark.parametrize("metric", ["cosine", "euclidean", "manhattan"])
def test_explicit_triplet(metric):
    a, p, n = _leaf(6, 5, seed=10), _leaf(6, 5, seed=11), _leaf(6, 5, seed=12)
    margin = 0.5 if metric == "cosine" else 3.0

    def d(x, y_):
        if metric == "cosine":
            return 1 - _cos(x, y_)
        diff = x - y_
        return diff.pow(2).sum().sqrt() if metric == "euclidean" else diff.abs().sum()

    def oracle(a, p, n):
        return sum(torch.clamp(d(a[i], p[i]) - d(a[i], n[i]) + margin, min=0) for i in range(6)) / 6

    _check(lambda x, y_, z: O.explicit_triplet_loss(x, y_, z, metric=metric, margin=margin), oracle, [a, p, n])


LABELS = torch.tensor([0, 0, 1, 1, 2, 2, 0, 1, 3])


def _pair_d(x, i, j, metric):
    if metric == "cosine":
        return 1 - _cos(x[i], x[j])
    sq = ((x[i] - x[j]) ** 2).sum()
    if metric == "squared_euclidean":
        return sq
    return sq.sqrt() if i != j else sq * 0


@pytest.mark.parametrize("metric", ["euclidean", "squared_euclidean", "cosine"])
def test_batch_all_triplet(metric):
    x = _leaf(9, 4, seed=13)
    margin = 1.0 if metric == "cosine" else 5.0

    def oracle(x):
        losses = []
        for a in range(9):
            for p in range(9):
                if p == a or LABELS[p] != LABELS[a]:
                    continue
                for n in range(9):
                    if LABELS[n] == LABELS[a]:
                        continue
                    value = _pair_d(x, a, p, metric) - _pair_d(x, a, n, metric) + margin
                    if float(value) > 1e-16:
                        losses.append(value)
        return sum(losses) / max(len(losses), 1)

    _check(lambda y: O.batch_all_triplet_loss(y, LABELS, metric=metric, margin=margin), oracle, [x])


@pytest.mark.parametrize("soft", [False, True])
def test_batch_hard_triplet_with_lonely_anchor(soft):
    """Label 3 has no positive: that anchor is skipped (reference semantics)."""

    x = _leaf(9, 4, seed=14)

    def oracle(x):
        rows = []
        for a in range(9):
            pos = [_pair_d(x, a, p, "euclidean") for p in range(9) if p != a and LABELS[p] == LABELS[a]]
            neg = [_pair_d(x, a, n, "euclidean") for n in range(9) if LABELS[n] != LABELS[a]]
            if not pos or not neg:
                continue
            hp = max(pos, key=float)
            hn = min(neg, key=float)
            rows.append(torch.log1p(torch.exp(hp - hn)) if soft else torch.clamp(hp - hn + 5.0, min=0))
        return sum(rows) / len(rows)

    impl = (lambda y: O.batch_hard_soft_margin_triplet_loss(y, LABELS)) if soft else (
        lambda y: O.batch_hard_triplet_loss(y, LABELS, margin=5.0))
    _check(impl, oracle, [x])


def test_batch_semi_hard_triplet():
    x = _leaf(9, 4, seed=15)

    def oracle(x):
        rows = []
        for a in range(9):
            negs = [n for n in range(9) if LABELS[n] != LABELS[a]]
            if not negs:
                continue
            for p in range(9):
                if p == a or LABELS[p] != LABELS[a]:
                    continue
                dap = _pair_d(x, a, p, "euclidean")
                farther = [_pair_d(x, a, n, "euclidean") for n in negs if float(_pair_d(x, a, n, "euclidean")) > float(dap)]
                chosen = min(farther, key=float) if farther else max(
                    (_pair_d(x, a, n, "euclidean") for n in negs), key=float)
                rows.append(torch.clamp(dap - chosen + 5.0, min=0))
        return sum(rows) / len(rows)

    _check(lambda y: O.batch_semi_hard_triplet_loss(y, LABELS, margin=5.0), oracle, [x])


# ------------------------------------------------------------------ distillation (K5)
@pytest.mark.parametrize("metric", ["mse", "l2", "cosine"])
def test_embedding_distillation(metric):
    s, t = _leaf(5, 6, seed=16), _leaf(5, 6, seed=17)
    t = t.detach()

    def oracle(s):
        rows = []
        for i in range(5):
            if metric == "mse":
                rows.append(((s[i] - t[i]) ** 2).mean())
            elif metric == "l2":
                rows.append((s[i] - t[i]).norm())
            else:
                rows.append(1 - _cos(s[i], t[i]))
        return sum(rows) / 5

    _check(lambda a: O.embedding_distillation_loss(a, t.float(), metric=metric), oracle, [s])


@pytest.mark.parametrize("similarity", ["dot", "cosine"])
def test_margin_mse(similarity):
    q, p, n = _leaf(6, 4, seed=18), _leaf(6, 4, seed=19), _leaf(6, 4, seed=20)
    margin = torch.randn(6, generator=torch.Generator().manual_seed(21), dtype=torch.float64)

    def oracle(q, p, n):
        total = 0
        for i in range(6):
            if similarity == "dot":
                m = q[i] @ p[i] - q[i] @ n[i]
            else:
                m = _cos(q[i], p[i]) - _cos(q[i], n[i])
            total = total + (m - margin[i]) ** 2
        return total / 6

    _check(lambda a, b, c: O.margin_mse_loss(a, b, c, margin.float(), similarity=similarity), oracle, [q, p, n])


def test_distribution_kl_with_temperature():
    s, t = _leaf(4, 5, seed=22), _leaf(4, 5, seed=23).detach()
    temp = 2.0

    def oracle(s):
        total = 0
        for i in range(4):
            ps = torch.softmax(s[i] / temp, 0)
            pt = torch.softmax(t[i] / temp, 0)
            total = total + sum(pt[j] * (torch.log(pt[j]) - torch.log(ps[j])) for j in range(5)) * temp ** 2
        return total / 4

    _check(lambda a: O.distribution_kl_loss(a, t.float(), temperature=temp), oracle, [s])


# ------------------------------------------------------------------ classification (K7)
@pytest.mark.parametrize("concat", [("u", "v", "abs_diff"), ("u", "v", "abs_diff", "mul")])
def test_softmax_classification(concat):
    u, v = _leaf(6, 4, seed=24), _leaf(6, 4, seed=25)
    w = _leaf(3, 4 * len(concat), seed=26)
    b = _leaf(3, seed=27)
    labels = torch.tensor([0, 2, 1, 1, 0, 2])

    def oracle(u, v, w, b):
        total = 0
        for i in range(6):
            parts = {"u": u[i], "v": v[i], "abs_diff": (u[i] - v[i]).abs(), "mul": u[i] * v[i]}
            feat = torch.cat([parts[k] for k in concat])
            logits = w @ feat + b
            total = total + torch.logsumexp(logits, 0) - logits[labels[i]]
        return total / 6

    _check(lambda a, c, ww, bb: O.softmax_classification_loss(a, c, labels, ww, bb, concatenation=concat)[0],
           oracle, [u, v, w, b])


# ------------------------------------------------------------------ contrastive tension (K8)
def test_contrastive_tension_pairs():
    u, v = _leaf(6, 4, seed=28), _leaf(6, 4, seed=29)
    y = torch.tensor([1, 0, 0, 1, 0, 0], dtype=torch.float64)

    def oracle(u, v):
        total = 0
        for i in range(6):
            z = u[i] @ v[i]
            total = total - (y[i] * torch.log(torch.sigmoid(z)) + (1 - y[i]) * torch.log(1 - torch.sigmoid(z)))
        return total / 6

    _check(lambda a, b: O.contrastive_tension_loss(a, b, y.float()), oracle, [u, v])


def test_contrastive_tension_in_batch():
    u, v = _leaf(5, 4, seed=30), _leaf(5, 4, seed=31)

    def oracle(u, v):
        s = [[_cos(u[i], v[j]) * 20.0 for j in range(5)] for i in range(5)]
        rows = sum(torch.logsumexp(torch.stack(s[i]), 0) - s[i][i] for i in range(5)) / 5
        cols = sum(torch.logsumexp(torch.stack([s[j][i] for j in range(5)]), 0) - s[i][i] for i in range(5)) / 5
        return (rows + cols) / 2

    _check(lambda a, b: O.contrastive_tension_in_batch_loss(a, b, scale=20.0), oracle, [u, v])


# ------------------------------------------------------------------ regularisation, mega-batch (K9, K11, T4)
def test_gor_weights():
    a, n = _leaf(8, 4, seed=32), _leaf(8, 4, seed=33)

    def oracle(a, n):
        dots = [_cos(a[i], n[i]) for i in range(8)]
        m1 = sum(dots) / 8
        m2 = sum(d ** 2 for d in dots) / 8
        return 0.5 * m1 ** 2 + 2.0 * torch.clamp(m2 - 1 / 4, min=0)

    _check(lambda x, y: O.global_orthogonal_regularization(x, y, mean_weight=0.5, second_moment_weight=2.0),
           oracle, [a, n])


def test_mega_batch_margin_and_hardest_negative():
    a, p, n = _leaf(6, 5, seed=34), _leaf(6, 5, seed=35), _leaf(6, 5, seed=36)

    def oracle(a, p, n):
        return sum(torch.clamp(0.8 - _cos(a[i], p[i]), min=0) + torch.clamp(_cos(a[i], n[i]) - 0.3, min=0)
                   for i in range(6)) / 6

    _check(lambda x, y, z: O.mega_batch_margin_loss(x, y, z), oracle, [a, p, n])
    idx = O.hardest_negative_indices(a.detach().float(), p.detach().float(), chunk=4)
    for i in range(6):
        scores = [float(_cos(a[i], p[j])) if j != i else -math.inf for j in range(6)]
        assert int(idx[i]) == max(range(6), key=lambda j: scores[j])


# ------------------------------------------------------------------ retrieval MNR (K2)
@pytest.mark.parametrize("symmetric", [False, True])
def test_mnr_reference_with_weights_and_validity(symmetric):
    from representax_b200.ops.mnr import mnr_terms_reference

    q, d = _leaf(5, 4, seed=37), _leaf(7, 4, seed=38)
    w = torch.zeros(5, 7, dtype=torch.float64)
    for i in range(5):
        w[i, i] = 1.0
    w[1, 6] = 0.5
    w[4, 4] = 0.0  # row 4 has no positive: inactive
    qv = torch.tensor([True, True, True, False, True])
    dv = torch.tensor([True, True, False, True, True, True, True])
    scale = 20.0

    def direction(rows, cands, ww, rv, cv):
        losses = []
        for i in range(rows.shape[0]):
            if not rv[i]:
                continue
            logits = [(_cos(rows[i], cands[j]) * scale, j) for j in range(cands.shape[0]) if cv[j]]
            weight = sum(float(ww[i, j]) for _, j in logits)
            if weight <= 0:
                continue
            lse = torch.logsumexp(torch.stack([l for l, _ in logits]), 0)
            term = sum(ww[i, j] * (lse - l) for l, j in logits if ww[i, j] > 0)
            losses.append(term / max(weight, 1.0))
        return sum(losses) / max(len(losses), 1)

    def oracle(q, d):
        f = direction(q, d, w, qv, dv)
        return (f + direction(d, q, w.T, dv, qv)) / 2 if symmetric else f

    _check(lambda a, b: mnr_terms_reference(a, b, w.float(), qv, dv, scale, symmetric)[0], oracle, [q, d])


# ------------------------------------------------------------------ GIST (K6)
@pytest.mark.parametrize("strategy,margin", [("absolute", 0.05), ("relative", 0.1)])
def test_gist_false_negative_filtering(strategy, margin):
    from representax_b200.tasks.guided import gist_loss_terms

    a, p = _leaf(5, 4, seed=39), _leaf(5, 4, seed=40)
    ga, gp = _leaf(5, 4, seed=41).detach(), _leaf(5, 4, seed=42).detach()
    ga[2] = gp[3] * 1.01  # a guide near-duplicate makes (2, 3) a filtered false negative
    temp = 0.05

    def oracle(a, p):
        total = 0
        for i in range(5):
            pos_guide = float(_cos(ga[i], gp[i]))
            limit = pos_guide - margin if strategy == "absolute" else pos_guide - abs(pos_guide) * margin
            cands = []
            for j in range(5):  # anchor-positive block: the positive plus unfiltered negatives
                g = float(_cos(ga[i], gp[j]))
                if j == i or g <= limit:
                    cands.append(_cos(a[i], p[j]) / temp)
            for j in range(5):  # anchor-anchor block
                if j != i and float(_cos(ga[i], ga[j])) <= limit:
                    cands.append(_cos(a[i], a[j]) / temp)
            for j in range(5):  # positive-positive block
                if j != i and float(_cos(gp[i], gp[j])) <= limit:
                    cands.append(_cos(p[i], p[j]) / temp)
            logits = torch.stack(cands)
            total = total + torch.logsumexp(logits, 0) - _cos(a[i], p[i]) / temp
        return total / 5

    def impl(x, y):
        return gist_loss_terms([x, y], [ga.float(), gp.float()], temperature=temp, margin_strategy=strategy,
                               margin=margin).loss

    _check(impl, oracle, [a, p], tol=dict(rtol=1e-4, atol=1e-5))


# ------------------------------------------------------------------ modifiers (K12)
class _PairTask:
    """Cosine-regression representation task on ready-made representations."""

    def __init__(self, labels):
        self.labels = labels

    def loss_from_representations(self, reps, batch):
        from representax_b200.core import LossOutput

        left, right = reps
        return LossOutput(loss=O.cosine_regression_loss(left, right, self.labels), metrics={})


def test_matryoshka_prefixes_and_weights():
    from representax_b200.tasks.modifiers import MatryoshkaTask

    u, v = _leaf(4, 8, seed=43), _leaf(4, 8, seed=44)
    y = torch.tensor([0.2, 0.8, 0.5, 0.1], dtype=torch.float64)
    dims, weights = (8, 4, 2), (1.0, 0.5, 2.0)

    def oracle(u, v):
        total = 0
        for dim, wt in zip(dims, weights):
            total = total + wt * sum((_cos(u[i, :dim], v[i, :dim]) - y[i]) ** 2 for i in range(4)) / 4
        return total

    task = MatryoshkaTask(_PairTask(y.float()), dims, weights=weights)
    _check(lambda a, b: task.loss_from_representations((a, b), None).loss, oracle, [u, v])


class _LayerModel(torch.nn.Module):
    """A fake layerwise encoder: fixed [layers, batch, dim] representations."""

    def __init__(self, layers):
        super().__init__()
        from representax_b200.core import EncoderMetadata

        self.layers = layers
        self.metadata = EncoderMetadata(model_id="fake", revision="1", output_dimension=layers.shape[-1])

    def encode(self, inputs, *, route, generator=None):
        return self.layers[-1][inputs]

    def encode_layers(self, inputs, *, route, generator=None):
        return self.layers[:, inputs]


class _LayerPairTask(_PairTask):
    def representations(self, model, batch, *, generator=None, encode_fn=None):
        from representax_b200.core import Route

        left = encode_fn(model, batch[0], route=Route.GENERIC)
        right = encode_fn(model, batch[1], route=Route.GENERIC)
        return left, right


def test_adaptive_layer_all_layers():
    from representax_b200.tasks.modifiers import AdaptiveLayerTask

    layers = _leaf(3, 8, 4, seed=45)
    y = torch.tensor([0.3, 0.9, 0.1, 0.6], dtype=torch.float64)
    batch = (torch.arange(0, 4), torch.arange(4, 8))
    temp = 0.3

    def cr(left, right):
        return sum((_cos(left[i], right[i]) - y[i]) ** 2 for i in range(4)) / 4

    def kl(teacher, student):
        t_all = torch.cat(teacher).detach()
        s_all = torch.cat(student)
        ts, ss = t_all @ t_all.T / temp, s_all @ s_all.T / temp
        total = 0
        for i in range(ts.shape[0]):
            pt, ps = torch.softmax(ts[i], 0), torch.softmax(ss[i], 0)
            total = total + (pt * (torch.log(pt) - torch.log(ps))).sum()
        return total / ts.shape[0] * temp * temp

    def oracle(layers):
        final = (layers[-1, :4], layers[-1, 4:])
        loss = cr(*final)
        for i in range(2):  # prior layers 0 and 1, both selected
            prior = (layers[i, :4], layers[i, 4:])
            loss = loss + (1 + i) / 2 * cr(*prior) / 2 + kl(final, prior) / 2
        return loss

    task = AdaptiveLayerTask(_LayerPairTask(y.float()), layers_per_step=-1, kl_temperature=temp)

    def impl(ls):
        from representax_b200.precision import FP32_POLICY, precision_context

        with precision_context(FP32_POLICY):
            return task.loss(_LayerModel(ls), batch).loss

    _check(impl, oracle, [layers], tol=dict(rtol=1e-4, atol=1e-5))


def test_matryoshka_2d_equals_adaptive_over_matryoshka():
    from representax_b200.precision import FP32_POLICY, precision_context
    from representax_b200.tasks.modifiers import AdaptiveLayerTask, Matryoshka2dTask, MatryoshkaTask

    layers = _leaf(3, 8, 8, seed=46).detach().float().requires_grad_(True)
    y = torch.tensor([0.3, 0.9, 0.1, 0.6])
    batch = (torch.arange(0, 4), torch.arange(4, 8))
    base = _LayerPairTask(y)
    joint = Matryoshka2dTask(base, dimensions=(8, 4), layers_per_step=-1)
    inner = MatryoshkaTask(base, (8, 4))

    class _Composed:
        def representations(self, *a, **k):
            return inner.representations(*a, **k)

        def loss_from_representations(self, reps, b):
            return inner.loss_from_representations(reps, b)

    composed = AdaptiveLayerTask(_Composed(), layers_per_step=-1)
    with precision_context(FP32_POLICY):
        a = joint.loss(_LayerModel(layers), batch).loss
        b = composed.loss(_LayerModel(layers), batch).loss
    assert torch.allclose(a, b, rtol=1e-6, atol=1e-7)
