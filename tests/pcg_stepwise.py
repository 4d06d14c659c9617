"""Preconditioned conjugate gradient on the explicit Schur system S.

Same iteration, stopping rule and return value as the reference's ``_pcg``
(inference/ba_solver.py:1197-1238): x0 = 0, Jacobi preconditioner, stop when
||r|| <= tol ||b|| (returning that iterate), break on a non-finite r.z (returning the
best-so-far iterate), else the best-so-far iterate after maxiter.  The reference syncs
the host on every iteration; here the state lives on the device and iterates that come
after the stopping event are masked out, so the host only checks every ``check_every``
iterations.  The operator is the library's block-sparse S matvec.
"""
import torch


def pcg(A_mv, b, M_mv=None, tol=1e-6, maxiter=300, check_every=16):
    dt = b.dtype
    x = torch.zeros_like(b)
    r = b - A_mv(x)
    z = M_mv(r) if M_mv is not None else r
    p = z.clone()
    rz_old = torch.dot(r, z)
    bnorm = torch.linalg.vector_norm(b).clamp(min=1e-12)
    best_norm = torch.full((), float('inf'), dtype=dt, device=b.device)
    best_x = x.clone()
    best_k = torch.zeros((), dtype=torch.int64, device=b.device)
    active = torch.ones((), dtype=torch.bool, device=b.device)
    converged = torch.zeros((), dtype=torch.bool, device=b.device)
    k_stop = torch.zeros((), dtype=torch.int64, device=b.device)
    for k in range(1, maxiter + 1):
        Ap = A_mv(p)
        denom = torch.dot(p, Ap).clamp(min=1e-32)
        alpha = torch.where(active, rz_old / denom, torch.zeros_like(denom))
        x = x + alpha * p
        r = r - alpha * Ap
        rn = torch.linalg.vector_norm(r)
        better = active & (rn < best_norm)
        best_norm = torch.where(better, rn, best_norm)
        best_x = torch.where(better, x, best_x)
        best_k = torch.where(better, torch.full_like(best_k, k), best_k)
        conv_now = active & (rn <= tol * bnorm)
        converged = converged | conv_now
        k_stop = torch.where(conv_now, torch.full_like(k_stop, k), k_stop)
        active = active & ~conv_now
        z = M_mv(r) if M_mv is not None else r
        rz_new = torch.dot(r, z)
        bad = active & ~torch.isfinite(rz_new)
        active = active & ~bad
        beta = rz_new / rz_old.clamp(min=1e-32)
        p = torch.where(active, z + beta * p, p)
        rz_old = torch.where(active, rz_new, rz_old)
        if k % check_every == 0 and not bool(active):
            break
    if bool(converged):
        return x, int(k_stop), True
    return best_x, int(best_k), False
