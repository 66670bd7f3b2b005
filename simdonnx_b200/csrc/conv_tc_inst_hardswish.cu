// conv_tc_kernel instantiations for the hardswish epilogue activation (one unit per activation so the
// kernels compile in parallel).
#include "conv_tc_kernel.cuh"

namespace sdx {
template int launch_tc<ACT_HARDSWISH, 4, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_HARDSWISH, 4, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_HARDSWISH, 1, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_HARDSWISH, 1, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_HARDSWISH, 2, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_HARDSWISH, 0, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_HARDSWISH, 0, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_HARDSWISH, 6, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
}  // namespace sdx
