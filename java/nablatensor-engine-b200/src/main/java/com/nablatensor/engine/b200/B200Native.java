/*
 * FFM (java.lang.foreign) binding of libnabla_b200.so, the B200 tape-replay
 * engine's C ABI (include/nabla_b200.h of the engine's repository).
 *
 * Every downcall returns 0 or a negative NT_E_* status; check() turns a
 * status into the exception the reference's engine SPI uses for it
 * (AadEngine.java:50-86, CudaRuntime.java:124-137), with the library's
 * thread-local message.  The library is found at
 * -Dnablatensor.b200.library, else as libnabla_b200.so on the loader path.
 * It is bound on first use from a holder class, so a machine without it can
 * still enumerate engines (AadEngine.isAvailable must never throw).
 */
package com.nablatensor.engine.b200;

import static java.lang.foreign.ValueLayout.ADDRESS;
import static java.lang.foreign.ValueLayout.JAVA_BYTE;
import static java.lang.foreign.ValueLayout.JAVA_DOUBLE;
import static java.lang.foreign.ValueLayout.JAVA_INT;
import static java.lang.foreign.ValueLayout.JAVA_LONG;

import java.lang.foreign.Arena;
import java.lang.foreign.FunctionDescriptor;
import java.lang.foreign.Linker;
import java.lang.foreign.MemoryLayout;
import java.lang.foreign.MemorySegment;
import java.lang.foreign.StructLayout;
import java.lang.foreign.SymbolLookup;
import java.lang.invoke.MethodHandle;
import java.nio.file.Path;

final class B200Native {
  private B200Native() {}

  // Status codes (nabla_b200.h).
  static final int NT_OK = 0;
  static final int NT_E_INVALID_ARG = -1;
  static final int NT_E_TAPE = -2;
  static final int NT_E_UNSUPPORTED = -3;
  static final int NT_E_STATE = -8;

  // Option flags (nabla_b200.h), keyed by the engine-option names
  // AadOptions.engineOptions("cuda") carries.
  static final int NT_FLAG_NO_LOOP = 0x1;
  static final int NT_FLAG_SHARED_CKPT = 0x2;
  static final int NT_FLAG_F32_FAST = 0x8;
  static final int NT_FLAG_NO_FMAD = 0x10;
  static final int NT_FLAG_RECOMPUTE_ALL = 0x40;
  static final int NT_FLAG_TAPE_DRAWS = 0x80;
  static final int NT_FLAG_TAPE_ALL = 0x100;

  /** struct nt_tape: the FlatTape arrays plus the per-stream draw counts. */
  static final StructLayout TAPE = MemoryLayout.structLayout(
      JAVA_INT.withName("n"), MemoryLayout.paddingLayout(4),
      ADDRESS.withName("op"), ADDRESS.withName("arg_a"), ADDRESS.withName("arg_b"), ADDRESS.withName("constant"),
      JAVA_INT.withName("n_in"), MemoryLayout.paddingLayout(4), ADDRESS.withName("input_node"),
      JAVA_INT.withName("n_out"), MemoryLayout.paddingLayout(4), ADDRESS.withName("output_node"),
      JAVA_INT.withName("n_streams"), MemoryLayout.paddingLayout(4),
      ADDRESS.withName("normal_count"), ADDRESS.withName("uniform_count"));

  /** struct nt_options: AadOptions plus the engine's tuning knobs (0 = automatic). */
  static final StructLayout OPTIONS = MemoryLayout.structLayout(
      JAVA_INT.withName("precision"), JAVA_INT.withName("adjoints"), JAVA_INT.withName("device"),
      JAVA_INT.withName("block"), JAVA_INT.withName("seg_units"), JAVA_INT.withName("min_blocks"),
      JAVA_INT.withName("max_regs"), JAVA_INT.withName("flags"), JAVA_INT.withName("fwd_unroll"),
      JAVA_INT.withName("grid_blocks_per_sm"), JAVA_INT.withName("rev_unroll"));

  /** The downcall handles, bound when first used. */
  static final class Api {
    private Api() {}

    private static final Linker LINKER = Linker.nativeLinker();
    private static final SymbolLookup LIB = SymbolLookup.libraryLookup(
        Path.of(System.getProperty("nablatensor.b200.library", "libnabla_b200.so")), Arena.global());

    private static MethodHandle fn(String name, FunctionDescriptor d) {
      return LINKER.downcallHandle(LIB.find(name).orElseThrow(
          () -> new UnsatisfiedLinkError("libnabla_b200.so has no symbol " + name)), d);
    }

    static final MethodHandle NT_VERSION = fn("nt_version", FunctionDescriptor.of(JAVA_INT));
    static final MethodHandle NT_LAST_ERROR = fn("nt_last_error", FunctionDescriptor.of(ADDRESS));
    static final MethodHandle NT_INIT = fn("nt_init", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle NT_COMPILE = fn("nt_compile",
        FunctionDescriptor.of(JAVA_INT, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle NT_SET_INPUTS = fn("nt_set_inputs",
        FunctionDescriptor.of(JAVA_INT, ADDRESS, ADDRESS, JAVA_INT));
    static final MethodHandle NT_REPLAY = fn("nt_replay",
        FunctionDescriptor.of(JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle NT_REPLAY_MARKETS = fn("nt_replay_markets",
        FunctionDescriptor.of(JAVA_INT, ADDRESS, JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, ADDRESS,
            ADDRESS));
    static final MethodHandle NT_REPLAY_ACCUMULATE = fn("nt_replay_accumulate",
        FunctionDescriptor.of(JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG));
    static final MethodHandle NT_ACCUMULATOR_READ = fn("nt_accumulator_read",
        FunctionDescriptor.of(JAVA_INT, ADDRESS, ADDRESS, JAVA_INT));
    static final MethodHandle NT_DESTROY = fn("nt_destroy", FunctionDescriptor.ofVoid(ADDRESS));
    static final MethodHandle NT_DIST_UNIQUE_ID = fn("nt_dist_unique_id", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle NT_DIST_ATTACH = fn("nt_dist_attach",
        FunctionDescriptor.of(JAVA_INT, ADDRESS, JAVA_INT, JAVA_INT, ADDRESS, JAVA_INT));
    static final MethodHandle NT_REPLAY_SHARDED = fn("nt_replay_sharded",
        FunctionDescriptor.of(JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle NT_DIST_DETACH = fn("nt_dist_detach", FunctionDescriptor.of(JAVA_INT, ADDRESS));
  }

  /** Wraps anything a downcall threw as an unchecked exception (the SPI declares none). */
  static RuntimeException unchecked(Throwable t) {
    if (t instanceof RuntimeException r) {
      return r;
    }
    if (t instanceof Error e) {
      throw e;
    }
    return new IllegalStateException("cuda engine: " + t, t);
  }

  /** The calling thread's last error message. */
  static String lastError() {
    try {
      MemorySegment s = (MemorySegment) Api.NT_LAST_ERROR.invokeExact();
      return s.reinterpret(4096).getString(0);
    } catch (Throwable t) {
      return "(no message: " + t + ")";
    }
  }

  /** A status as the SPI's exceptions: arguments, unsupported tapes, state, and the rest. */
  static void check(int rc) {
    if (rc == NT_OK) {
      return;
    }
    String msg = lastError();
    switch (rc) {
      case NT_E_INVALID_ARG, NT_E_TAPE -> throw new IllegalArgumentException(msg);
      case NT_E_UNSUPPORTED -> throw new UnsupportedOperationException(msg);
      case NT_E_STATE -> throw new IllegalStateException(msg);
      default -> throw new IllegalStateException("cuda engine (status " + rc + "): " + msg);
    }
  }

  /** CUDA devices visible to the engine (0 without a driver or device). */
  static int deviceCount() {
    try (Arena a = Arena.ofConfined()) {
      MemorySegment n = a.allocate(JAVA_INT);
      check((int) Api.NT_INIT.invokeExact(n));
      return n.get(JAVA_INT, 0);
    } catch (Throwable t) {
      throw unchecked(t);
    }
  }

  /** 128-byte NCCL unique id for rank 0 to broadcast to the others. */
  static byte[] uniqueId() {
    try (Arena a = Arena.ofConfined()) {
      MemorySegment id = a.allocate(128);
      check((int) Api.NT_DIST_UNIQUE_ID.invokeExact(id));
      return id.toArray(JAVA_BYTE);
    } catch (Throwable t) {
      throw unchecked(t);
    }
  }
}
