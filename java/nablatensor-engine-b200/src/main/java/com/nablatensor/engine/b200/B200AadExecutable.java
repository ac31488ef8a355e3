/*
 * One compiled tape on one B200: AadExecutable for engine "cuda"
 * (AadExecutable.java:37-78) on top of AbstractAadExecutable's chunking,
 * calibration and input bookkeeping (AbstractAadExecutable.java:36-165).
 *
 * replay(paths, pathOffset, seed) issues as many device launches as the
 * reference's dispatch budget needs (GpuAadExecutable.maxLaunchSeconds, so no
 * single kernel outlives a display watchdog), accumulates their sums exactly
 * on the device (nt_replay_accumulate) and reads them back once
 * (nt_accumulator_read).  Launches start on 32-scenario tile boundaries, so
 * the result has the same bits as one launch over the whole range.
 */
package com.nablatensor.engine.b200;

import static java.lang.foreign.ValueLayout.ADDRESS;
import static java.lang.foreign.ValueLayout.JAVA_BYTE;
import static java.lang.foreign.ValueLayout.JAVA_DOUBLE;
import static java.lang.foreign.ValueLayout.JAVA_INT;

import com.nablatensor.engine.AadOptions;
import com.nablatensor.engine.AadResult;
import com.nablatensor.engine.AadTape;
import com.nablatensor.engine.AadTotals;
import com.nablatensor.engine.AbstractAadExecutable;
import com.nablatensor.engine.FlatTape;
import com.nablatensor.engine.GpuAadExecutable;
import java.lang.foreign.Arena;
import java.lang.foreign.MemoryLayout.PathElement;
import java.lang.foreign.MemorySegment;
import java.lang.foreign.StructLayout;
import java.util.Map;

public final class B200AadExecutable extends AbstractAadExecutable {
  /** Paths of one warp tile: every launch after the first starts on a multiple of it. */
  private static final long TILE = 32L;
  /** Paths per launch until a rate has been measured. */
  private static final long FIRST_LAUNCH_PATHS = 1L << 22;
  private static final long MIN_LAUNCH_PATHS = 65_536L;

  private final MemorySegment handle;
  private final int channels;
  private final double compileSeconds;
  private final double launchSeconds;
  private double launchPathsPerSecond;
  private boolean accumulatorDirty;
  private boolean released;

  B200AadExecutable(AadTape tape, AadOptions options) {
    super(tape, options);
    this.channels = tape.outputCount() * (2 + tape.inputCount());
    this.launchSeconds = GpuAadExecutable.maxLaunchSeconds(2.0);
    long t0 = System.nanoTime();
    try (Arena a = Arena.ofConfined()) {
      MemorySegment out = a.allocate(ADDRESS);
      B200Native.check((int) B200Native.Api.NT_COMPILE.invokeExact(marshalTape(a, tape), marshalOptions(a, options),
          out));
      this.handle = out.get(ADDRESS, 0);
    } catch (Throwable t) {
      throw B200Native.unchecked(t);
    }
    this.compileSeconds = (System.nanoTime() - t0) * 1e-9;
  }

  /**
   * FlatTape (FlatTape.java:37-79) as struct nt_tape: op ordinals
   * (AadOpEnum order), both argument arrays, constants, input and output
   * nodes, and the per-stream normal and uniform draw counts
   * (AadTape.java:128-196).  The library copies every array during
   * nt_compile, so they live in the caller's confined arena.
   */
  private static MemorySegment marshalTape(Arena a, AadTape tape) {
    FlatTape f = new FlatTape(tape);
    int n = f.size();
    int[] op = new int[n];
    for (int i = 0; i < n; i++) {
      op[i] = f.op[i].ordinal();
    }
    int streams = f.randStreams;
    int[] normals = new int[streams];
    int[] uniforms = new int[streams];
    for (int s = 0; s < streams; s++) {
      normals[s] = tape.randNormalCount(s);
      uniforms[s] = tape.randUniformCount(s);
    }
    StructLayout l = B200Native.TAPE;
    MemorySegment t = a.allocate(l);
    t.set(JAVA_INT, off(l, "n"), n);
    t.set(ADDRESS, off(l, "op"), a.allocateFrom(JAVA_INT, op));
    t.set(ADDRESS, off(l, "arg_a"), a.allocateFrom(JAVA_INT, f.argA));
    t.set(ADDRESS, off(l, "arg_b"), a.allocateFrom(JAVA_INT, f.argB));
    t.set(ADDRESS, off(l, "constant"), a.allocateFrom(JAVA_DOUBLE, f.constant));
    t.set(JAVA_INT, off(l, "n_in"), f.inputNode.length);
    t.set(ADDRESS, off(l, "input_node"), f.inputNode.length > 0 ? a.allocateFrom(JAVA_INT, f.inputNode)
        : MemorySegment.NULL);
    t.set(JAVA_INT, off(l, "n_out"), f.outputNode.length);
    t.set(ADDRESS, off(l, "output_node"), a.allocateFrom(JAVA_INT, f.outputNode));
    t.set(JAVA_INT, off(l, "n_streams"), streams);
    t.set(ADDRESS, off(l, "normal_count"), streams > 0 ? a.allocateFrom(JAVA_INT, normals) : MemorySegment.NULL);
    t.set(ADDRESS, off(l, "uniform_count"), streams > 0 ? a.allocateFrom(JAVA_INT, uniforms) : MemorySegment.NULL);
    return t;
  }

  /**
   * AadOptions as struct nt_options: precision ordinal (FLOAT32 = 0,
   * FLOAT64 = 1), adjoints, and the knobs of engineOptions("cuda") -- the
   * same keys the engine's Python mirror accepts; an unknown key is an
   * IllegalArgumentException.
   */
  private static MemorySegment marshalOptions(Arena a, AadOptions options) {
    StructLayout l = B200Native.OPTIONS;
    MemorySegment o = a.allocate(l);
    o.set(JAVA_INT, off(l, "precision"), options.precision().ordinal());
    o.set(JAVA_INT, off(l, "adjoints"), options.adjoints() ? 1 : 0);
    int flags = 0;
    for (Map.Entry<String, String> e : options.engineOptions("cuda").entrySet()) {
      String v = e.getValue();
      boolean on = "1".equals(v) || "true".equalsIgnoreCase(v) || "on".equalsIgnoreCase(v);
      switch (e.getKey()) {
        case "device" -> o.set(JAVA_INT, off(l, "device"), Integer.parseInt(v));
        case "block" -> o.set(JAVA_INT, off(l, "block"), Integer.parseInt(v));
        case "segUnits" -> o.set(JAVA_INT, off(l, "seg_units"), Integer.parseInt(v));
        case "minBlocks" -> o.set(JAVA_INT, off(l, "min_blocks"), Integer.parseInt(v));
        case "maxRegs" -> o.set(JAVA_INT, off(l, "max_regs"), Integer.parseInt(v));
        case "fwdUnroll" -> o.set(JAVA_INT, off(l, "fwd_unroll"), Integer.parseInt(v));
        case "gridBlocksPerSm" -> o.set(JAVA_INT, off(l, "grid_blocks_per_sm"), Integer.parseInt(v));
        case "revUnroll" -> o.set(JAVA_INT, off(l, "rev_unroll"), Integer.parseInt(v));
        case "noLoop" -> flags |= on ? B200Native.NT_FLAG_NO_LOOP : 0;
        case "sharedCheckpoints" -> flags |= on ? B200Native.NT_FLAG_SHARED_CKPT : 0;
        case "fp32Fast" -> flags |= on ? B200Native.NT_FLAG_F32_FAST : 0;
        case "noFmad" -> flags |= on ? B200Native.NT_FLAG_NO_FMAD : 0;
        case "recomputeAll" -> flags |= on ? B200Native.NT_FLAG_RECOMPUTE_ALL : 0;
        case "tapeDraws" -> flags |= on ? B200Native.NT_FLAG_TAPE_DRAWS : 0;
        case "tapeAll" -> flags |= on ? B200Native.NT_FLAG_TAPE_ALL : 0;
        default -> throw new IllegalArgumentException("unknown cuda engine option: " + e.getKey());
      }
    }
    o.set(JAVA_INT, off(l, "flags"), flags);
    return o;
  }

  private static long off(StructLayout l, String field) {
    return l.byteOffset(PathElement.groupElement(field));
  }

  /**
   * replaySafe's chunk budget.  calibrate() grows its probe dispatches eight
   * times over until one takes a fifth of the budget, and a B200 replays
   * about 1e9 scenarios a second: the reference's 2 s budget would spend some
   * 2 s of probes before the first real chunk, while each further chunk costs
   * only a launch and a 56-byte read-back.  So the budget is short (20 ms,
   * -Dnablatensor.b200.maxChunkSeconds to change), and never longer than the
   * reference's dispatch budget -Dnablatensor.maxLaunchSeconds when that is
   * set.  Called from the base constructor: it reads system properties only.
   */
  @Override
  protected double defaultMaxChunkSeconds() {
    double chunk = Double.parseDouble(System.getProperty("nablatensor.b200.maxChunkSeconds", "0.02"));
    return Math.min(chunk, GpuAadExecutable.maxLaunchSeconds(Double.MAX_VALUE));
  }

  @Override
  public String engineName() {
    return "cuda";
  }

  @Override
  public double compileSeconds() {
    return compileSeconds;
  }

  /** One replay of [pathOffset, pathOffset + paths) in launches of at most the dispatch budget. */
  @Override
  public AadResult replay(long paths, long pathOffset, long seed) {
    checkOpen();
    if (paths <= 0) {
      throw new IllegalArgumentException("paths must be positive");
    }
    long t0 = System.nanoTime();
    try (Arena a = Arena.ofConfined()) {
      MemorySegment sums = a.allocate(JAVA_DOUBLE, channels);
      if (accumulatorDirty) {  // an earlier replay failed between its launches and its read-back
        B200Native.check((int) B200Native.Api.NT_ACCUMULATOR_READ.invokeExact(handle, sums, 1));
        accumulatorDirty = false;
      }
      MemorySegment in = a.allocateFrom(JAVA_DOUBLE, inputs);
      B200Native.check((int) B200Native.Api.NT_SET_INPUTS.invokeExact(handle, in, inputs.length));
      long step = launchPaths();
      accumulatorDirty = true;
      for (long done = 0; done < paths; done += step) {
        long k = Math.min(step, paths - done);
        B200Native.check((int) B200Native.Api.NT_REPLAY_ACCUMULATE.invokeExact(handle, k, pathOffset + done, seed));
      }
      B200Native.check((int) B200Native.Api.NT_ACCUMULATOR_READ.invokeExact(handle, sums, 1));
      accumulatorDirty = false;
      double seconds = (System.nanoTime() - t0) * 1e-9;
      if (seconds > 0.0) {
        double rate = paths / seconds;
        launchPathsPerSecond = launchPathsPerSecond <= 0.0 ? rate : 0.5 * (launchPathsPerSecond + rate);
      }
      return totals(sums, 0).toResult(tape, paths, seconds);
    } catch (Throwable t) {
      throw B200Native.unchecked(t);
    }
  }

  /** Scenarios per device launch: the measured rate times the dispatch budget, whole tiles. */
  private long launchPaths() {
    if (launchPathsPerSecond <= 0.0) {
      return FIRST_LAUNCH_PATHS;
    }
    long k = (long) Math.min(Long.MAX_VALUE / 2, launchPathsPerSecond * launchSeconds);
    return Math.max(MIN_LAUNCH_PATHS, k - k % TILE);
  }

  /** The sums of one channel block ([sum v, sum v^2, sum adjoints] per output) as AadTotals. */
  private AadTotals totals(MemorySegment sums, long base) {
    AadTotals t = new AadTotals(tape.outputCount(), tape.inputCount());
    long k = base;
    for (int o = 0; o < tape.outputCount(); o++) {
      t.value[o] = sums.getAtIndex(JAVA_DOUBLE, k++);
      t.sumsq[o] = sums.getAtIndex(JAVA_DOUBLE, k++);
      for (int j = 0; j < tape.inputCount(); j++) {
        t.gradient[o][j] = sums.getAtIndex(JAVA_DOUBLE, k++);
      }
    }
    return t;
  }

  /**
   * Re-pricing under several markets in one dispatch with common random
   * numbers (nt_replay_markets): the per-market loop of ScenarioRunner.run /
   * ladder (nablatensor-quant/.../scenario/ScenarioRunner.java:36-71) without a
   * replay per market.  markets[m] is a full input vector in input order.
   */
  public AadResult[] replayMarkets(double[][] markets, long paths, long pathOffset, long seed) {
    checkOpen();
    if (paths <= 0) {
      throw new IllegalArgumentException("paths must be positive");
    }
    int nIn = tape.inputCount();
    long t0 = System.nanoTime();
    try (Arena a = Arena.ofConfined()) {
      MemorySegment in = a.allocate(JAVA_DOUBLE, (long) markets.length * Math.max(1, nIn));
      for (int m = 0; m < markets.length; m++) {
        if (markets[m].length != nIn) {
          throw new IllegalArgumentException("market " + m + " has " + markets[m].length + " inputs, expected " + nIn);
        }
        MemorySegment.copy(markets[m], 0, in, JAVA_DOUBLE, (long) m * nIn * 8, nIn);
      }
      MemorySegment sums = a.allocate(JAVA_DOUBLE, (long) markets.length * channels);
      MemorySegment secs = a.allocate(JAVA_DOUBLE);
      B200Native.check((int) B200Native.Api.NT_REPLAY_MARKETS.invokeExact(handle, markets.length, in, paths,
          pathOffset, seed, sums, secs));
      double seconds = (System.nanoTime() - t0) * 1e-9;
      AadResult[] out = new AadResult[markets.length];
      for (int m = 0; m < markets.length; m++) {
        out[m] = totals(sums, (long) m * channels).toResult(tape, paths, seconds);
      }
      return out;
    } catch (Throwable t) {
      throw B200Native.unchecked(t);
    }
  }

  /** 128-byte NCCL unique id; rank 0 creates it and hands it to the other ranks. */
  public static byte[] distUniqueId() {
    return B200Native.uniqueId();
  }

  /** Joins an nranks-wide communicator (one process per GPU); timeoutMs bounds every wait. */
  public void distAttach(int nranks, int rank, byte[] uniqueId, int timeoutMs) {
    checkOpen();
    if (uniqueId.length != 128) {
      throw new IllegalArgumentException("the unique id has 128 bytes");
    }
    try (Arena a = Arena.ofConfined()) {
      MemorySegment id = a.allocateFrom(JAVA_BYTE, uniqueId);
      B200Native.check((int) B200Native.Api.NT_DIST_ATTACH.invokeExact(handle, nranks, rank, id, timeoutMs));
    } catch (Throwable t) {
      throw B200Native.unchecked(t);
    }
  }

  /**
   * This rank's contiguous shard of [pathOffset, pathOffset + totalPaths) and
   * one all-reduce: every rank gets the global result, with the same bits as
   * a single-GPU replay of the whole range.
   */
  public AadResult replaySharded(long totalPaths, long pathOffset, long seed, long chunkPaths) {
    checkOpen();
    if (totalPaths <= 0) {
      throw new IllegalArgumentException("paths must be positive");
    }
    try (Arena a = Arena.ofConfined()) {
      MemorySegment in = a.allocateFrom(JAVA_DOUBLE, inputs);
      B200Native.check((int) B200Native.Api.NT_SET_INPUTS.invokeExact(handle, in, inputs.length));
      MemorySegment sums = a.allocate(JAVA_DOUBLE, channels);
      MemorySegment secs = a.allocate(JAVA_DOUBLE);
      B200Native.check((int) B200Native.Api.NT_REPLAY_SHARDED.invokeExact(handle, totalPaths, pathOffset, seed,
          chunkPaths, sums, secs));
      return totals(sums, 0).toResult(tape, totalPaths, secs.get(JAVA_DOUBLE, 0));
    } catch (Throwable t) {
      throw B200Native.unchecked(t);
    }
  }

  /** Leaves the communicator. */
  public void distDetach() {
    checkOpen();
    try {
      B200Native.check((int) B200Native.Api.NT_DIST_DETACH.invokeExact(handle));
    } catch (Throwable t) {
      throw B200Native.unchecked(t);
    }
  }

  /** Releases the device state once; later calls fail in checkOpen() (AbstractAadExecutable.java:94-98). */
  @Override
  public void close() {
    if (!released) {
      released = true;
      try {
        B200Native.Api.NT_DESTROY.invokeExact(handle);
      } catch (Throwable ignored) {
        // nothing to recover: the handle is gone either way
      }
    }
    super.close();
  }
}
