// pdl.cuh -- programmatic dependent launch between consecutive kernels.
//
// Every kernel of the library is launched with programmatic stream
// serialisation allowed and starts with HX_PDL_PROLOGUE(), a
// griddepcontrol.wait: it returns once every grid this one depends on has
// completed and its writes are visible (a no-op without a dependency).
// No kernel triggers its dependents early, so the next kernel of the stream
// is launched as the CTAs of this one exit (the implicit trigger) instead of
// after the whole grid has drained and its completion has reached the host
// queue: its launch overlaps this kernel's tail and memory flush.
//
// Measured on B200 (one step of the tiny-Transformer LM, CUDA graph; A =
// T64 D48 F48 L4 H4 with Muon, 32 sequences; B = T64 D64 F64 L2 H4 with Adam,
// 16 sequences; C = T256 D256 F1024 L4 H8, 64 sequences):
//   no PDL                                     A 763 us, B 325 us, C 3.678 ms
//   wait + launch_dependents at kernel entry   A 844 us, B 324 us, C 3.643 ms
//   wait only (this prologue)                  A 717-725 us, B 312 us, C 3.622 ms
// An entry trigger lets the next kernel's CTAs sit resident, waiting, on the
// SMs the side stream's weight-gradient GEMMs would use, which costs more than
// the launch latency it hides.
//
// Because every kernel waits before its first instruction, completion is
// transitive along the stream: kernel k+2 may read what kernel k wrote.
// The wait comes before anything else, so no CTA holds tensor memory or
// spins on a barrier while a grid it depends on is still running.
#pragma once

#define HX_PDL_PROLOGUE() asm volatile("griddepcontrol.wait;" ::: "memory")
