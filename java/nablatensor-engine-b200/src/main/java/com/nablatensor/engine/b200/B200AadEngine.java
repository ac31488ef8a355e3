/*
 * Engine "cuda" on B200: the AadEngine SPI (AadEngine.java:28-48) over
 * libnabla_b200.so.  Registered through
 * META-INF/services/com.nablatensor.engine.AadEngine; with priority 110 it is
 * found before nablatensor-engine-cuda's CudaAadEngine (priority 100) when
 * both are on the class path (AadEngines.find takes the first name match in
 * priority order, AadEngines.java:67-74), so
 * MonteCarlo.of(...).greeks().on("cuda") selects it unchanged.
 */
package com.nablatensor.engine.b200;

import com.nablatensor.engine.AadEngine;
import com.nablatensor.engine.AadExecutable;
import com.nablatensor.engine.AadOptions;
import com.nablatensor.engine.AadTape;

public final class B200AadEngine implements AadEngine {
  /** The engine's priority; nablatensor_b200.engine.CudaAadEngine answers the same. */
  static final int PRIORITY = 110;

  @Override
  public String name() {
    return "cuda";
  }

  @Override
  public int priority() {
    return PRIORITY;
  }

  /** A loadable library and at least one device; never throws (AadEngine.java:39-40). */
  @Override
  public boolean isAvailable() {
    try {
      return B200Native.deviceCount() > 0;
    } catch (Throwable t) {
      return false;
    }
  }

  /** fp32 (the reference's fp32 semantics) and fp64 both run. */
  @Override
  public boolean supports(AadOptions options) {
    return options.precision() == AadOptions.PrecisionEnum.FLOAT32
        || options.precision() == AadOptions.PrecisionEnum.FLOAT64;
  }

  @Override
  public String describe() {
    return "B200 sm_100a · NVRTC tape kernels · fp32+fp64";
  }

  /**
   * Multi-output tapes, uniform draws and named random streams are replayed
   * natively, so unlike the reference's generated-kernel engines this one
   * does not call requireSupportedTape.
   */
  @Override
  public AadExecutable compile(AadTape tape, AadOptions options) {
    if (!isAvailable()) {
      throw new IllegalStateException("no CUDA device available for the B200 replay kernel");
    }
    return new B200AadExecutable(tape, options);
  }
}
