"""The forward's device memory: one libqdc_b200 workspace arena per model.

Replaces the reference's per-model ForwardWorkspace (ext/cuda_workspace.jl:
4-87): there every intermediate of a forward is a `scratch(T, dims)` slot,
reused by call order, the cursor reset at the start of each forward
(native_forward_scope, :48-69) and per layer kind (:279-300), and a captured
graph replays the slots it was recorded against (:241-259).  Here the slots
are carved from the context's arena (qdc_ws_alloc) in call order:

  begin(nbytes)   start of a forward: make sure the arena holds `nbytes`
                  (growing it reallocates, so `generation` moves on and every
                  graph recorded against the old arena must be dropped), and
                  reset the cursor to 0;
  take(shape)     the next slot, as a tensor view of arena memory (no torch
                  allocation); the same call order gives the same addresses,
                  forward after forward;
  mark()/release(m)  the cursor before a layer and back to it after, so every
                  layer carves the same slots as the one before it.

A slot is valid until the next begin(); callers copy results out before the
model's next forward (the reference reads back inside native_forward_scope
for the same reason, src/backbone.jl:440-452)."""
import torch

GROWTH = 1.5  # a growing arena takes at least this factor more, so growth events stay few
MAX_VIEWS = 4096  # cached slot views (a forward carves a few hundred)


class Workspace:
    def __init__(self, ctx):
        self.ctx = ctx
        self.device = ctx.device
        self.generation = 0
        self._base = None
        self._views = {}  # (offset, shape, dtype) -> cached view: slots reused by call order

    @property
    def capacity(self):
        return self.ctx.ws_stats()[1]

    def begin(self, nbytes):
        """Start a forward that carves at most `nbytes`."""
        cap = self.capacity
        if nbytes > cap:
            self.ctx.ws_reserve(max(int(nbytes), int(cap * GROWTH)))
            self.generation += 1
            self._views.clear()
            self._base = None
        self.ctx.ws_reset()
        if self._base is None:
            self._base = self.ctx.ws_alloc(1)
            self.ctx.ws_reset()

    def take(self, shape, dtype=torch.float32):
        """The next slot of `shape` (a tensor view of arena memory)."""
        shape = tuple(int(s) for s in shape)
        numel = 1
        for s in shape:
            numel *= s
        nbytes = max(numel * _itemsize(dtype), 1)
        ptr = self.ctx.ws_alloc(nbytes)
        key = (ptr - self._base, shape, dtype)
        view = self._views.get(key)
        if view is None:
            if len(self._views) >= MAX_VIEWS:  # many shapes seen: start over
                self._views.clear()
            view = self._views[key] = self.ctx.wrap(ptr, shape, dtype)
        return view

    def take_all(self, spec):
        """Slots for every entry of `spec` (name -> (shape, dtype)), in order."""
        return {name: self.take(shape, dtype) for name, (shape, dtype) in spec.items()}

    def mark(self):
        return self.ctx.ws_mark()

    def release(self, mark):
        self.ctx.ws_release(mark)

    def contains(self, t):
        """Whether tensor `t`'s storage lies inside the arena."""
        cap = self.capacity
        p = t.data_ptr()
        return self._base is not None and self._base <= p < self._base + cap


_ITEMSIZE = {}


def _itemsize(dtype):
    size = _ITEMSIZE.get(dtype)
    if size is None:
        size = _ITEMSIZE[dtype] = torch.empty((), dtype=dtype).element_size()
    return size


def spec_bytes(spec):
    """Arena bytes of take_all(spec)."""
    return sum(slot_bytes(shape, dtype) for shape, dtype in spec.values())


def slot_bytes(shape, dtype=torch.float32):
    """Arena bytes of one take(shape, dtype): the size rounded up to the
    arena's 256-byte alignment."""
    numel = 1
    for s in shape:
        numel *= int(s)
    return (max(numel * _itemsize(dtype), 1) + 255) // 256 * 256
