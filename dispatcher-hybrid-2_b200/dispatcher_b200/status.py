"""The device status word that every bounded wait in the kernels reports to.

A kernel whose wait on a TMA copy, an mbarrier or another CTA's flag runs
past its limit writes DH_ERR_TIMEOUT (a bad token id writes DH_ERR_ARG) into
an int32 on the device and returns instead of hanging; its output is then
wrong.  `StatusWord` turns that into a Python exception without putting a
host synchronisation on the launch path: `arm()` queues an asynchronous copy
of the word into pinned host memory behind the launches just issued, and
`check()` raises `DispatcherB200Error` once that copy has landed with a
nonzero value (at the next call, or at once with `sync=True`).  The word is
cleared when it is reported, so the next call starts clean.
"""

import torch

from ._lib import ERRORS, DispatcherB200Error


class StatusWord:
    def __init__(self, device):
        self.device = torch.device(device)
        self.tensor = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._event = None

    def data_ptr(self):
        return self.tensor.data_ptr()

    def arm(self):
        """Queue the read-back of the word behind the work issued so far on
        the current stream."""
        self._host.copy_(self.tensor, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._event = ev

    def check(self, where, sync=False):
        """Raise if a read-back that has completed (or, with sync, the pending
        one) saw a nonzero word."""
        ev = self._event
        if ev is None:
            return
        if sync:
            ev.synchronize()
        elif not ev.query():
            return
        self._event = None
        code = int(self._host[0])
        if code != 0:
            self.tensor.zero_()
            self._host.zero_()
            raise DispatcherB200Error(
                where, code,
                f"a kernel reported {ERRORS.get(code, code)} on the device (a bounded wait "
                f"gave up or an input was out of range); the results of that call are invalid")
