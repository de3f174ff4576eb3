"""Host-array steps streamed through the device.

The reference's host entry points (``gpu_matmul``, src/gpu.rs:98-169, and the
gpu_step calls behind it) upload, compute and download one call at a time.
``HostPipeline`` runs a sequence of such steps with the three phases on
their own CUDA streams: while step i computes, step i+1's inputs go up and
step i-1's results come down (PCIe is full duplex, and the copy engines run
beside the SMs).  ``depth`` device buffer sets alternate: a set's inputs are
refilled once its previous compute has finished reading them, and it is
computed into again once its previous results have been downloaded, so in
the steady state a step costs the slowest of the three phases.  Each set's compute is
captured once into a CUDA graph, so a step costs the host one graph launch
and one ``cudaMemcpyAsync`` per tensor.
"""
import torch


class HostPipeline:
    """``sets[j] = (inputs, outputs)``: the device tensors a step of buffer set
    j reads and writes; ``run(j)`` enqueues set j's compute on torch's current
    stream (it must not allocate, synchronise, or read host memory, so that
    it can be captured).  ``submit(host_inputs, host_outputs)`` enqueues one
    step and returns its ticket; host tensors should be pinned, and a step's
    ``host_outputs`` must not be reused before ``wait`` on its ticket."""

    def __init__(self, sets, run, device, graphs=True):
        self.device = torch.device(device)
        self.sets = sets
        self.up = torch.cuda.Stream(self.device)
        self.comp = torch.cuda.Stream(self.device)
        self.down = torch.cuda.Stream(self.device)
        self.consumed = [None] * len(sets)  # set j's last compute has finished
        self.free = [None] * len(sets)      # set j's last results are downloaded
        self.run = run
        self.graphs = None
        for j in range(len(sets)):  # eager run first: grows scratch, sets kernel attributes
            with torch.cuda.stream(self.comp):
                run(j)
        torch.cuda.synchronize(self.device)
        if graphs:
            self.graphs = []
            for j in range(len(sets)):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=self.comp):
                    run(j)
                self.graphs.append(g)
            torch.cuda.synchronize(self.device)
        self.i = 0

    def submit(self, host_inputs, host_outputs):
        """Enqueues one step; returns its ticket (a CUDA event)."""
        j = self.i % len(self.sets)
        self.i += 1
        inputs, outputs = self.sets[j]
        if len(host_inputs) != len(inputs) or len(host_outputs) != len(outputs):
            raise ValueError("a step takes %d inputs and %d outputs" % (len(inputs), len(outputs)))
        if self.consumed[j] is not None:
            self.up.wait_event(self.consumed[j])
        with torch.cuda.stream(self.up):
            for dst, src in zip(inputs, host_inputs):
                dst.copy_(torch.as_tensor(src), non_blocking=True)
        ready = torch.cuda.Event()
        ready.record(self.up)
        self.comp.wait_event(ready)
        if self.free[j] is not None:
            self.comp.wait_event(self.free[j])
        with torch.cuda.stream(self.comp):
            if self.graphs is not None:
                self.graphs[j].replay()
            else:
                self.run(j)
        done = torch.cuda.Event()
        done.record(self.comp)
        self.consumed[j] = done
        self.down.wait_event(done)
        with torch.cuda.stream(self.down):
            for dst, src in zip(host_outputs, outputs):
                dst.copy_(src, non_blocking=True)
        ticket = torch.cuda.Event()
        ticket.record(self.down)
        self.free[j] = ticket
        return ticket

    @staticmethod
    def wait(ticket):
        ticket.synchronize()

    def close(self):
        """Waits for every step in flight and releases the graphs."""
        torch.cuda.synchronize(self.device)
        self.graphs = None
