"""Single-process data parallelism for research jobs on the GPUs of one lease.

One persistent model replica per device.  An update splits the global rows over the replicas in
order (uneven shares allowed), each replica runs its micro-batches forward and backward, the
gradients are summed into the first replica in fp32 weighted by row counts (so the update equals
one device's update on the whole batch), the optimizer steps once there, and the new parameters
are copied to the other replicas.  Data order and row identities do not depend on the device
count.  This is the research path of the reference gym (``gym/src/nexttransformer_gym/research.py``),
not the formal trainer: the formal trainer is one process per GPU over NCCL.
"""
import copy

import torch


class ResearchDP:
    def __init__(self, model, devices, make_optimizer):
        self.devices = [torch.device(d) for d in devices]
        if not self.devices:
            raise ValueError("at least one device")
        self.replicas = [model.to(self.devices[0])]
        for d in self.devices[1:]:
            self.replicas.append(copy.deepcopy(model).to(d))
        self.optimizer = make_optimizer(self.replicas[0])
        self._params = [list(r.parameters()) for r in self.replicas]

    def shares(self, rows):
        """Rows of each replica: contiguous, in order, as even as possible."""
        n = len(self.replicas)
        base, extra = divmod(rows, n)
        return [base + (1 if i < extra else 0) for i in range(n)]

    def step(self, x, y, micro_rows, loss_fn):
        """One update on ``x``, ``y`` [rows, T] (host or device tensors); returns the mean loss."""
        rows = x.shape[0]
        total_loss = 0.0
        start = 0
        for replica, params, dev, share in zip(self.replicas, self._params, self.devices, self.shares(rows)):
            for p in params:
                p.grad = None
            for m0 in range(start, start + share, micro_rows):
                m1 = min(m0 + micro_rows, start + share)
                xb, yb = x[m0:m1].to(dev, non_blocking=True), y[m0:m1].to(dev, non_blocking=True)
                loss = loss_fn(replica, xb, yb)
                # each micro-batch weighs its rows in the global mean
                (loss * ((m1 - m0) / rows)).backward()
                total_loss += float(loss.detach()) * (m1 - m0) / rows
            start += share
        main = self._params[0]
        for others in self._params[1:]:
            for p0, p in zip(main, others):
                if p.grad is None:
                    continue
                g = p.grad.detach().to(p0.device, dtype=torch.float32)
                if p0.grad is None:
                    p0.grad = g.to(p0.dtype)
                else:
                    p0.grad = (p0.grad.float() + g).to(p0.dtype)
        self.optimizer.step()
        self.optimizer.zero_grad(set_to_none=True)
        with torch.no_grad():
            for others in self._params[1:]:
                for p0, p in zip(main, others):
                    p.copy_(p0.detach().to(p.device))
        return total_loss
