// Layout of the NVLink peer-memory exchange used for tensor-parallel sums of decode-sized messages.
//
// Every rank owns one receive buffer, mapped into every other rank (CUDA IPC over NVLink/NVSwitch):
//   [call counters: kP2pCtas ints, padded to kP2pHeader bytes]
//   [slots: 2 parities x world sources x kP2pCapacity values x 8 bytes]
// A value travels as ONE 8-byte store {float bits, call epoch}: the receiver polls the values
// themselves until their epoch is the current one, so no fence or flag is needed. The epoch of a
// call is (counter + 1); the exchange kernels always run kP2pCtas CTAs and CTA g keeps counter g, so
// every counter holds the number of completed calls between calls, with no atomics. Parity =
// epoch & 1: a rank writes slot parity p again only two calls later, after every other rank has
// pushed the intervening call, which each does only after its own receive of this call finished.
#pragma once

#include <cstddef>
#include <cstdint>

namespace shd {

constexpr int kP2pMaxWorld = 8;
constexpr int kP2pCtas = 16;                        // CTAs of every exchange launch (fixed)
constexpr int kP2pThreads = 512;
constexpr size_t kP2pHeader = 256;                  // call counters, then slots
constexpr size_t kP2pCapacity = 2 * 8 * 8192;       // values: both shares of 8 rows x 8192
constexpr size_t kP2pSlotBytes = kP2pCapacity * 8;  // {value, epoch} pairs
static_assert(kP2pCtas * 4 <= (int)kP2pHeader, "call counters fit the header");

// Slot (parity, source) of a receive buffer.
__host__ __device__ __forceinline__ unsigned long long* p2p_slot(uint8_t* buf, int parity, int world, int source) {
  return reinterpret_cast<unsigned long long*>(buf + kP2pHeader + ((size_t)parity * world + source) * kP2pSlotBytes);
}

}  // namespace shd
