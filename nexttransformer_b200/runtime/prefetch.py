"""Background packing of the next micro-batches of a data stream.

``PrefetchStream(stream, depth)`` wraps a ``BestFitStream`` or ``SyntheticStream``: a thread reads
the parquet row groups, tokenises, packs (the C++ best-fit packer) and pins the next ``depth``
batches while the GPU runs the current one; ``batch()`` only issues the non-blocking host-to-device
copies.  Checkpoints stay exact: each queued batch carries the stream state after it, and
``state_dict()`` is the state after the last batch handed out, not after the last one packed.  A
different batch size, or ``load_state_dict``, stops the thread, rewinds the stream to that state
and starts again, so the rows a trainer sees never depend on the prefetch depth.
"""
import copy
import queue
import threading

import torch


class PrefetchStream:
    def __init__(self, stream, depth=2):
        if depth < 1:
            raise ValueError("prefetch depth must be at least 1")
        self.stream, self.depth = stream, depth
        self._state = stream.state_dict()
        self._rows = stream.rows
        self._queue, self._thread, self._stop, self._size, self._pin = None, None, None, None, False

    def __getattr__(self, name):  # identity, tokenizer, paths, ...
        return getattr(self.__dict__["stream"], name)

    @property
    def rows(self):
        """Rows handed out so far (the wrapped stream has packed further ahead)."""
        return self._rows

    def _produce(self, q, stop, size, pin):
        try:
            while not stop.is_set():
                x, y = self.stream.cpu_batch(size, pin=pin)
                item = (x, y, self.stream.state_dict(), self.stream.rows)
                while not stop.is_set():
                    try:
                        q.put(item, timeout=0.05)
                        break
                    except queue.Full:
                        pass
        except BaseException as e:  # handed to the consumer, raised there
            while not stop.is_set():
                try:
                    q.put(e, timeout=0.05)
                    break
                except queue.Full:
                    pass

    def _start(self, size, pin):
        self._queue, self._stop = queue.Queue(maxsize=self.depth), threading.Event()
        self._size, self._pin = size, pin
        self._thread = threading.Thread(target=self._produce, args=(self._queue, self._stop, size, pin),
                                        name="nt-prefetch", daemon=True)
        self._thread.start()

    def close(self):
        """Stop the thread and rewind the stream to the state after the last batch handed out."""
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
            self._thread = None
            self.stream.load_state_dict(self._state)

    def batch(self, batch_size, device):
        pin = torch.device(device).type == "cuda"
        if self._thread is not None and (batch_size != self._size or pin != self._pin):
            self.close()
        if self._thread is None:
            self._start(batch_size, pin)
        item = self._queue.get()
        if isinstance(item, BaseException):
            self._thread.join()
            self._thread = None
            raise item
        x, y, self._state, self._rows = item
        return x.to(device, non_blocking=True), y.to(device, non_blocking=True)

    def batches(self, batch_size, device):
        while True:
            yield self.batch(batch_size, device)

    def state_dict(self):
        return copy.deepcopy(self._state)

    def load_state_dict(self, state):
        self.close()
        self.stream.load_state_dict(state)
        self._state = self.stream.state_dict()
        self._rows = self.stream.rows

    def __del__(self):
        try:
            if self._thread is not None:
                self._stop.set()
        except Exception:
            pass
