"""CPU restatement of torch-sla's Krylov hot path (test infrastructure only).

Each function names the torch-sla source lines whose algorithm it restates.
All arithmetic uses the PyTorch CPU ops the reference uses, in the same
order, so iteration counts and residual histories match the reference.
"""
from __future__ import annotations

import math

import torch


# --------------------------------------------------------------- matrices
def csr(val, row, col, shape):
    """COO -> torch sparse CSR, coalescing duplicates
    (backends/pytorch_backend.py:138-142)."""
    idx = torch.stack([row.to(torch.int64), col.to(torch.int64)])
    return torch.sparse_coo_tensor(idx, val, tuple(shape)).to_sparse_csr()


def diagonal(val, row, col, n):
    """Sum of the diagonal COO entries (pytorch_backend.py:167-174)."""
    d = torch.zeros(n, dtype=val.dtype)
    m = row == col
    d.scatter_add_(0, row[m].to(torch.int64), val[m])
    return d


def jacobi_inverse(d, rule: str):
    """'eps' (pytorch_backend.py:221-235), 'clamp' (distributed/solve.py:95-115),
    'nonzero' (pytorch_backend.py:2611-2614)."""
    if rule == "eps":
        eps = torch.finfo(d.dtype).eps * 100
        return 1.0 / torch.where(torch.abs(d) < eps, torch.ones_like(d), d)
    if rule == "clamp":
        return 1.0 / d.clamp_min(1e-30)
    if rule == "nonzero":
        return torch.where(d.abs() > 0, 1.0 / d, torch.ones_like(d))
    raise ValueError(rule)


def spmv(val, row, col, shape, x):
    """y = A x on the coalesced CSR (torch.mv, pytorch_backend.py:161)."""
    return torch.mv(csr(val, row, col, shape), x)


# ---------------------------------------------------------------- PCG
def pcg(val, row, col, shape, b, *, x0=None, atol=1e-10, rtol=1e-6, maxiter=10000,
        precond="jacobi"):
    """pcg_solve_fused + pcg_solve_optimized (pytorch_backend.py:1262-1362,
    1466-1501). Returns (x, iterations, residual, converged)."""
    A = csr(val, row, col, shape)
    n = shape[0]
    dinv = None if precond == "none" else jacobi_inverse(diagonal(val, row, col, n), "eps")
    apply_m = (lambda v: v) if dinv is None else (lambda v: dinv * v)
    if x0 is None:
        x = torch.zeros(n, dtype=b.dtype)
        r = b.clone()
    else:
        x = x0.clone()
        r = b - torch.mv(A, x)
    z = apply_m(r).clone()
    p = z.clone()
    rz = torch.vdot(r, z)
    tol_sq = max(atol, rtol * torch.norm(b).item()) ** 2
    for i in range(maxiter):
        rr = torch.vdot(r, r).real
        if rr.item() < tol_sq:  # start-of-iteration test
            return x, i, rr.sqrt().item(), True
        Ap = torch.mv(A, p)
        alpha = rz / torch.vdot(p, Ap)
        x.addcmul_(alpha, p)
        r.addcmul_(-alpha, Ap)
        z = apply_m(r).clone()
        rz_next = torch.vdot(r, z)
        beta = rz_next / rz
        p.mul_(beta).add_(z)
        rz = rz_next
    res = torch.norm(r).item()
    return x, maxiter, res, res < math.sqrt(tol_sq)


def pcg_mixed(val, row, col, shape, b, *, x0=None, atol=1e-10, rtol=1e-6, maxiter=10000,
              precond="jacobi"):
    """pytorch_solve's float32 + mixed_precision branch (pytorch_backend.py:
    2278-2285) into pcg_solve_mixed_precision (:1176-1255) with
    MixedPrecisionMatrix (:1143-1173). precond 'jacobi' / 'none' is the
    float32 preconditioner pytorch_solve wraps in M_f64 (r rounded to
    float32, result widened); 'default' is the float64 Jacobi the function
    builds when called without one (:1211-1216). Returns (x float64,
    iterations, residual, converged, p'Ap of a p'Ap <= 0 stop or None)."""
    n = shape[0]
    A32 = csr(val.to(torch.float32), row, col, shape)

    def mv(v):
        return torch.mv(A32, v.to(torch.float32)).to(torch.float64)

    if precond == "default":
        d64 = torch.zeros(n, dtype=torch.float64)
        m = row == col
        d64.scatter_add_(0, row[m].to(torch.int64), val[m].to(torch.float64))
        dinv64 = jacobi_inverse(d64, "eps")
        apply_m = lambda v: dinv64 * v  # noqa: E731
    else:
        if precond == "none":
            m32 = lambda v: v  # noqa: E731
        else:
            dinv32 = jacobi_inverse(diagonal(val.to(torch.float32), row, col, n), "eps")
            m32 = lambda v: dinv32 * v  # noqa: E731
        apply_m = lambda v: m32(v.to(torch.float32)).to(torch.float64)  # noqa: E731
    if x0 is None:
        x = torch.zeros(n, dtype=torch.float64)
        r = b.to(torch.float64).clone()
    else:
        x = x0.to(torch.float64).clone()
        r = b.to(torch.float64) - mv(x)
    z = apply_m(r)
    p = z.clone()
    rz_old = torch.vdot(r, z)
    b_norm = torch.norm(b.to(torch.float64))
    if b_norm == 0:
        b_norm = 1.0
    tol = max(atol, rtol * b_norm)
    residual = torch.norm(r).item()
    for i in range(maxiter):
        Ap = mv(p)
        pAp = torch.vdot(p, Ap)
        if pAp <= 0:
            return x, i, residual, False, float(pAp)
        alpha = rz_old / pAp
        x.add_(p, alpha=alpha.item())
        r.add_(Ap, alpha=-alpha.item())
        residual = torch.norm(r).item()
        if residual < tol:
            return x, i + 1, residual, True, None
        z = apply_m(r)
        rz_new = torch.vdot(r, z)
        beta = rz_new / rz_old
        p.mul_(beta.item()).add_(z)
        rz_old = rz_new
    return x, maxiter, residual, False, None


def csr_diagonal(A):
    """Diagonal of a torch CPU CSR matrix."""
    crow, colv, vals = A.crow_indices(), A.col_indices(), A.values()
    rows = torch.repeat_interleave(torch.arange(A.shape[0]), crow[1:] - crow[:-1])
    d = torch.zeros(A.shape[0], dtype=vals.dtype)
    m = rows == colv
    d.index_add_(0, rows[m], vals[m])
    return d


def pcg_iterations(A, b, dinv, iterations=None, budget_s=None):
    """Timed CPU sample: the loop body of pcg_solve_optimized
    (pytorch_backend.py:1317-1354) on a prebuilt CSR, for a fixed number of
    iterations or until `budget_s` seconds have passed. Returns the count."""
    import time
    x = torch.zeros_like(b)
    r = b.clone()
    z = (dinv * r).clone()
    p = z.clone()
    rz = torch.vdot(r, z)
    t0 = time.perf_counter()
    done = 0
    while True:
        if iterations is not None and done >= iterations:
            break
        if budget_s is not None and done > 0 and time.perf_counter() - t0 > budget_s:
            break
        torch.vdot(r, r).real.item()
        Ap = torch.mv(A, p)
        alpha = rz / torch.vdot(p, Ap)
        x.addcmul_(alpha, p)
        r.addcmul_(-alpha, Ap)
        z.copy_(dinv * r)
        rz_next = torch.vdot(r, z)
        p.mul_(rz_next / rz).add_(z)
        rz = rz_next
        done += 1
    return done


# ----------------------------------------------------------- BiCGStab
def pbicgstab(val, row, col, shape, b, *, x0=None, atol=1e-10, rtol=1e-6, maxiter=10000,
              precond="jacobi"):
    """pbicgstab_solve (pytorch_backend.py:1508-1596). Returns
    (x, iterations, residual, exit) with exit in {'converged_half',
    'converged', 'rho', 'tt', 'omega', 'maxiter'}; breakdowns and maxiter
    report `maxiter` iterations, as the reference does."""
    A = csr(val, row, col, shape)
    n = shape[0]
    dinv = None if precond == "none" else jacobi_inverse(diagonal(val, row, col, n), "eps")
    apply_m = (lambda v: v) if dinv is None else (lambda v: dinv * v)
    if x0 is None:
        x = torch.zeros(n, dtype=b.dtype)
        r = b.clone()
    else:
        x = x0.clone()
        r = b - torch.mv(A, x)
    rhat = r.clone()
    one = torch.tensor(1.0, dtype=b.dtype)
    rho_prev, alpha, omega = one, one, one
    v = torch.zeros(n, dtype=b.dtype)
    p = torch.zeros(n, dtype=b.dtype)
    bn = torch.norm(b)
    if bn == 0:
        bn = 1.0
    tol = max(atol, rtol * bn)
    residual = torch.norm(r).item()
    how = "maxiter"
    for i in range(maxiter):
        rho = torch.vdot(rhat, r)
        if abs(rho.item()) < 1e-30:
            how = "rho"
            break
        beta = (rho / rho_prev) * (alpha / omega)
        p = r + beta * (p - omega * v)
        ph = apply_m(p)
        v = torch.mv(A, ph)
        alpha = rho / torch.vdot(rhat, v)
        s = r - alpha * v
        sn = torch.norm(s).item()
        if sn < tol:
            return x + alpha * ph, i + 1, sn, "converged_half"
        sh = apply_m(s)
        t = torch.mv(A, sh)
        tt = torch.vdot(t, t).real
        if tt < 1e-30:
            x = x + alpha * ph
            how = "tt"
            break
        omega = torch.vdot(t, s) / tt
        x = x + alpha * ph + omega * sh
        r = s - omega * t
        residual = torch.norm(r).item()
        if residual < tol:
            return x, i + 1, residual, "converged"
        if abs(omega.item()) < 1e-30:
            how = "omega"
            break
        rho_prev = rho
    return x, maxiter, residual, how


# ------------------------------------------------------ batched CG
def batched_cg_same_pattern(val_batch, row, col, shape, b_batch, *, atol=1e-10, rtol=1e-6,
                            maxiter=10000):
    """batched_cg_same_pattern (pytorch_backend.py:2575-2638). Returns
    (X [B, n], iterations executed)."""
    n = shape[0]
    Bn = val_batch.shape[0]
    row = row.to(torch.int64)
    col = col.to(torch.int64)

    def matvec(X):
        Y = torch.zeros(Bn, n, dtype=val_batch.dtype)
        Y.index_add_(1, row, val_batch * X[:, col])
        return Y

    D = torch.zeros(Bn, n, dtype=val_batch.dtype)
    dm = row == col
    D.index_add_(1, row[dm], val_batch[:, dm])
    Dinv = torch.where(D.abs() > 0, 1.0 / D, torch.ones_like(D))
    X = torch.zeros(Bn, n, dtype=val_batch.dtype)
    R = b_batch.clone()
    Z = Dinv * R
    P = Z.clone()
    rz = (R * Z).sum(dim=1)
    tol = torch.clamp(rtol * torch.linalg.vector_norm(b_batch, dim=1).clamp_min(1e-30), min=atol)
    tiny = torch.tensor(1e-30, dtype=val_batch.dtype)
    it = 0
    for it in range(1, maxiter + 1):
        AP = matvec(P)
        pAp = (P * AP).sum(dim=1)
        alpha = rz / torch.where(pAp.abs() > 0, pAp, tiny)
        X = X + alpha.unsqueeze(1) * P
        R = R - alpha.unsqueeze(1) * AP
        if bool((torch.linalg.vector_norm(R, dim=1) <= tol).all()):
            break
        Z = Dinv * R
        rz_next = (R * Z).sum(dim=1)
        beta = rz_next / torch.where(rz.abs() > 0, rz, tiny)
        P = Z + beta.unsqueeze(1) * P
        rz = rz_next
    return X, it


# ------------------------------------------------------ multi-RHS CG
def batched_pcg(val, row, col, shape, B, *, X0=None, atol=1e-10, rtol=1e-6, maxiter=10000,
                dinv=None, check_interval=50):
    """batched_pcg_solve (pytorch_backend.py:2352-2504) with a column-wise
    diagonal preconditioner `dinv` ([n]) or none. Returns
    (X, num_iters [K], residuals [K], converged [K])."""
    A = csr(val, row, col, shape)
    n, K = B.shape
    apply_m = (lambda R: R) if dinv is None else (lambda R: dinv.unsqueeze(1) * R)
    if X0 is None:
        X = torch.zeros(n, K, dtype=B.dtype)
        R = B.clone()
    else:
        X = X0.clone()
        R = B - torch.mm(A, X)
    Z = apply_m(R)
    P = Z.clone()
    rz = (R * Z).sum(dim=0)
    bn = torch.norm(B, dim=0)
    bn = torch.where(bn == 0, torch.ones_like(bn), bn)
    tols = torch.maximum(torch.full_like(bn, atol), rtol * bn)
    tols_sq = tols ** 2
    conv = torch.zeros(K, dtype=torch.bool)
    iters = torch.zeros(K, dtype=torch.int32)
    for i in range(maxiter):
        if bool(conv.all()):
            break
        AP = torch.mm(A, P) if K > 1 else torch.mv(A, P.squeeze(1)).unsqueeze(1)
        PAP = (P * AP).sum(dim=0)
        PAP = torch.where(PAP > 0, PAP, torch.ones_like(PAP))
        alpha = rz / PAP
        X = X + alpha.unsqueeze(0) * P
        R = R - alpha.unsqueeze(0) * AP
        if (i + 1) % check_interval == 0:
            new = ((R * R).sum(dim=0) < tols_sq) & ~conv
            iters[new] = i + 1
            conv = conv | new
            if bool(conv.all()):
                break
        Z = apply_m(R)
        rz_next = (R * Z).sum(dim=0)
        P = Z + (rz_next / (rz + 1e-30)).unsqueeze(0) * P
        rz = rz_next
    res = torch.norm(R, dim=0)
    iters[~conv] = maxiter
    conv = conv | (res < tols)
    return X, iters, res, conv


# -------------------------------------------------------- adjoints
def adjoint(val, row, col, shape, u, gradu, *, method="cg", atol=1e-10, rtol=1e-10,
            maxiter=10000, precond="jacobi", mixed_precision=False):
    """SparseLinearSolvePyTorch.backward (linear_solve.py:303-324):
    A^T gradb = gradu on the swapped pattern, gradval = -gradb[row]*u[col].
    With mixed_precision (float32 CG) the adjoint solve is the mixed PCG and
    gradb is cast back to the value dtype (linear_solve.py:319-320)."""
    if mixed_precision and method == "cg" and val.dtype == torch.float32:
        fn = pcg_mixed
    else:
        fn = pcg if method == "cg" else pbicgstab
    gradb = fn(val, col, row, (shape[1], shape[0]), gradu, atol=atol, rtol=rtol,
               maxiter=maxiter, precond=precond)[0]
    gradb = gradb.to(val.dtype)
    gradval = -gradb[row.to(torch.int64)] * u[col.to(torch.int64)]
    return gradval, gradb


def batched_adjoint(val_batch, row, col, shape, u_batch, gradu_batch, *, atol=1e-10, rtol=1e-6,
                    maxiter=10000):
    """BatchSparseLinearSolveSameLayout.backward, CG branch (batch_solve.py:133-139)."""
    gradb = batched_cg_same_pattern(val_batch, col, row, (shape[1], shape[0]), gradu_batch,
                                    atol=atol, rtol=rtol, maxiter=maxiter)[0]
    gradval = -gradb[:, row.to(torch.int64)] * u_batch[:, col.to(torch.int64)]
    return gradval, gradb


# ----------------------------------------------- Shard(0) control flow
def cg_shard(val, row, col, shape, b, *, atol=1e-10, rtol=0.0, maxiter=1000, precond="jacobi",
             check_every=10):
    """cg_shard (distributed/solve.py:279-350) on the global vectors: the
    row-sharded solve computes the same recurrences, only its dot products are
    summed per rank first. Jacobi uses the clamp rule of make_preconditioner.
    Returns (x, iterations)."""
    A = csr(val, row, col, shape)
    n = shape[0]
    dinv = None if precond in (None, "none") else jacobi_inverse(diagonal(val, row, col, n), "clamp")
    apply_m = (lambda v: v) if dinv is None else (lambda v: dinv * v)
    x = torch.zeros_like(b)
    r = b - torch.mv(A, x)
    z = apply_m(r)
    p = z.clone()
    rs = torch.dot(r, z)
    tol = max(atol, rtol * float(torch.dot(b, b).sqrt().item()))
    iters = maxiter
    for k in range(maxiter):
        Ap = torch.mv(A, p)
        alpha = rs / torch.dot(p, Ap)
        torch.addcmul(x, alpha, p, value=1.0, out=x)
        torch.addcmul(r, alpha, Ap, value=-1.0, out=r)
        z = apply_m(r)
        rr, rs_next = torch.dot(r, r), torch.dot(r, z)
        if k % check_every == 0 and float(rr.sqrt().item()) < tol:
            iters = k + 1
            break
        p.mul_(rs_next / rs).add_(z)
        rs = rs_next
    return x, iters


def bicgstab_shard(val, row, col, shape, b, *, atol=1e-10, rtol=0.0, maxiter=1000,
                   precond="jacobi", check_every=10):
    """bicgstab_shard (distributed/solve.py:356-436) on the global vectors.
    Returns (x, iterations)."""
    A = csr(val, row, col, shape)
    n = shape[0]
    dinv = None if precond in (None, "none") else jacobi_inverse(diagonal(val, row, col, n), "clamp")
    apply_m = (lambda v: v) if dinv is None else (lambda v: dinv * v)
    x = torch.zeros_like(b)
    r = b - torch.mv(A, x)
    rhat = r.clone()
    rho = alpha = omega = torch.tensor(1.0, dtype=b.dtype)
    p = torch.zeros_like(b)
    v = torch.zeros_like(b)
    tol = max(atol, rtol * float(torch.dot(b, b).sqrt().item()))
    for k in range(maxiter):
        rho_k = torch.dot(rhat, r)
        p = r.clone() if k == 0 else r + (rho_k / rho) * (alpha / omega) * (p - omega * v)
        ph = apply_m(p)
        v = torch.mv(A, ph)
        alpha = rho_k / torch.dot(rhat, v)
        s = r - alpha * v
        ss = torch.dot(s, s)
        if k % check_every == 0 and float(ss.sqrt().item()) < tol:
            return x + alpha * ph, k + 1
        sh = apply_m(s)
        t = torch.mv(A, sh)
        # shard_matvec returns a view of one cached output buffer
        # (distributed/matvec.py:296-303), so computing t overwrites v: the
        # next iteration's p-update reads t where the textbook reads v.
        v = t
        omega = torch.dot(t, s) / torch.dot(t, t)
        x = x + alpha * ph + omega * sh
        r = s - omega * t
        if k % check_every == 0:
            rn = float(torch.dot(r, r).sqrt().item())
            if rn < tol or math.isnan(rn):
                return x, k + 1
        rho = rho_k
    return x, maxiter
