"""Training-step engine: the public per-update call of the framework.

``Trainer(model, optimizer, accumulation).step(inputs, targets)`` runs one optimizer update:
micro-batches are copied host->device (pinned, non-blocking), forward/backward through the
model (the fused sm_100a path on CUDA), gradients reduced to their owners and the Muon/AdamW
update applied by the optimizer, then the mean loss is read back to the host.
"""
import torch

from nexttransformer_b200.optim.groups import set_schedule
from nexttransformer_b200.utils.trace import nvtx_range


class Trainer:
    def __init__(self, model, optimizer, accumulation=1, train_config=None, schedule=True):
        self.model = model
        self.optimizer = optimizer
        self.accumulation = accumulation
        self.train_config = train_config
        self.schedule = schedule and train_config is not None
        self.step_index = 0
        self.device = model.get_device()
        # optional per-phase CUDA events of each update (``timing = True``): forward+backward of
        # all micro-batches, then the optimizer step; read with ``phase_times()`` after a sync
        self.timing = False
        self._events = []

    def zero_grad(self):
        m = self.model
        if hasattr(m, "zero_main_grads") and getattr(m, "_fused", None) is not None:
            m.zero_main_grads()
        for p in m.parameters():
            p.grad = None

    def step_device(self, inputs, targets):
        """One update on device-resident micro-batches ``inputs[i], targets[i]``; returns the loss tensor."""
        if self.schedule:
            set_schedule(self.optimizer, self.step_index, self.train_config)
        marks = None
        if self.timing and self.device.type == "cuda":
            marks = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            marks[0].record()
        self.zero_grad()
        total = torch.zeros((), device=self.device, dtype=torch.float32)
        st = getattr(self.model, "_fused", None)
        n = len(inputs)
        for j, (x, y) in enumerate(zip(inputs, targets)):
            if st is not None:
                st.final_micro = j == n - 1    # the last backward may start the gradient reductions
            with nvtx_range(f"micro{j}.forward"):
                loss = self.model(x, y)
            with nvtx_range(f"micro{j}.backward"):
                (loss / self.accumulation).backward()
            total += loss.detach().float()
        if st is not None:
            st.final_micro = False
        if marks is not None:
            marks[1].record()
        with nvtx_range("optimizer.step"):
            self.optimizer.step()
        if marks is not None:
            marks[2].record()
            self._events.append(marks)
        if hasattr(self.model, "update_router_bias"):
            self.model.update_router_bias()     # MoE aux-loss-free balancing, once per update
        self.step_index += 1
        return total / self.accumulation

    def phase_times(self, reset=True):
        """[(forward+backward ms, optimizer ms)] of the updates timed since the last call (the
        optimizer phase includes waiting for the gradient reductions it needs)."""
        out = [(a.elapsed_time(b), b.elapsed_time(c)) for a, b, c in self._events]
        if reset:
            self._events = []
        return out

    def flush(self):
        """Wait (on the current stream) for the parameter gathers the last update left running
        under the next forward; call before reading parameters outside the training step."""
        flush = getattr(self.optimizer, "flush", None)
        if flush is not None:
            flush()

    def step(self, inputs, targets):
        """One update from host (pinned) micro-batches; returns the mean loss as a Python float."""
        dev = self.device
        xs = [x.to(dev, non_blocking=True) for x in inputs]
        ys = [y.to(dev, non_blocking=True) for y in targets]
        return float(self.step_device(xs, ys))
